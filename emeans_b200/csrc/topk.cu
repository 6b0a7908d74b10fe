// Exact k-nearest rows by inner product (Device::topk, core/mod.rs:114-124):
// every score is one sequential FMA chain over d (the top-1 float order), and
// each query keeps the best kk by (larger score, then lower id), as knn_cpu
// does (crates/emeans-core/src/knn.rs:53-107): a candidate enters only when
// strictly better than the current last, so NaN and -inf never enter and
// missing neighbours stay (0xFFFFFFFF, -inf).
#include <cuda_runtime.h>

#include <algorithm>

#include "engine.h"

namespace eb {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256, KMAX = 16;

// Block (x, y): queries 64 x .. 64 x + 63 against data rows of chunk y,
// y chunk .. min(n, (y + 1) chunk) (all rows when gridDim.y is 1), whose
// global ids start at id0. Chunk y's lists go to out_ids / out_sims + y per.
// With exclude_self, query qi is skipped against the data row whose global
// id is qids[qi] (qi when qids is null).
__global__ void __launch_bounds__(NT) k_topk_exact(const float* __restrict__ q, long m,
                                                   const float* __restrict__ data_all, long n_all,
                                                   int d, int kk, int exclude_self, long id0,
                                                   const uint32_t* __restrict__ qids, long chunk,
                                                   long per, uint32_t* __restrict__ out_ids_all,
                                                   float* __restrict__ out_sims_all) {
  const long c0 = (long)blockIdx.y * chunk;
  const float* data = data_all + c0 * (long)d;
  const long n = gridDim.y == 1 ? n_all : min(chunk, n_all - c0);
  uint32_t* out_ids = out_ids_all + (long)blockIdx.y * per;
  float* out_sims = out_sims_all + (long)blockIdx.y * per;
  id0 += c0;
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  __shared__ float S[BM][BN + 1];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const long q0 = (long)blockIdx.x * BM;
  const int lr = tid >> 2, lc = (tid & 3) * 4;
  const bool a_live = q0 + lr < m;
  const float* arow = q + (a_live ? q0 + lr : 0) * (long)d;
  const bool vec = (d & 3) == 0;

  // Per-query list (threads 0..63 own query q0 + tid), best first.
  float ls[KMAX];
  uint32_t li[KMAX];
#pragma unroll
  for (int i = 0; i < KMAX; i++) {
    ls[i] = -INFINITY;
    li[i] = 0xFFFFFFFFu;
  }

  for (long n0 = 0; n0 < n; n0 += BN) {
    const bool b_live = n0 + lr < n;
    const float* brow = data + (b_live ? n0 + lr : 0) * (long)d;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < d; k0 += BK) {
      float av[4], bv[4];
      if (vec && k0 + lc + 4 <= d) {
        float4 a4 = a_live ? __ldg(reinterpret_cast<const float4*>(arow + k0 + lc))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 b4 = b_live ? __ldg(reinterpret_cast<const float4*>(brow + k0 + lc))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        av[0] = a4.x; av[1] = a4.y; av[2] = a4.z; av[3] = a4.w;
        bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
      } else {
#pragma unroll
        for (int t = 0; t < 4; t++) {
          int c = k0 + lc + t;
          av[t] = (a_live && c < d) ? __ldg(arow + c) : 0.0f;
          bv[t] = (b_live && c < d) ? __ldg(brow + c) : 0.0f;
        }
      }
#pragma unroll
      for (int t = 0; t < 4; t++) {
        As[lc + t][lr] = av[t];
        Bs[lc + t][lr] = bv[t];
      }
      __syncthreads();
      const int kmax = min(BK, d - k0);
      for (int kx = 0; kx < kmax; kx++) {
        float4 a4 = *reinterpret_cast<const float4*>(&As[kx][ty * 4]);
        float4 b4 = *reinterpret_cast<const float4*>(&Bs[kx][tx * 4]);
        float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) S[ty * 4 + i][tx * 4 + j] = acc[i][j];
    __syncthreads();
    if (tid < BM) {
      const long qi = q0 + tid;
      const long qg = q0 + tid < m ? (qids ? (long)qids[q0 + tid] : qi) : -1;
      int cols = (int)min((long)BN, n - n0);
      for (int j = 0; j < cols; j++) {
        // Data row n0 + j has the global id id0 + n0 + j (a shard's offset).
        uint32_t col = (uint32_t)(id0 + n0 + j);
        if (exclude_self && (long)col == qg) continue;
        float v = S[tid][j];
        if (!(v > ls[KMAX - 1])) continue;
        float cv = v;
        uint32_t cj = col;
#pragma unroll
        for (int i = 0; i < KMAX; i++) {
          bool b = cv > ls[i] || (cv == ls[i] && cj < li[i]);
          float tv = ls[i];
          uint32_t tj = li[i];
          ls[i] = b ? cv : tv;
          li[i] = b ? cj : tj;
          cv = b ? tv : cv;
          cj = b ? tj : cj;
        }
      }
    }
    __syncthreads();
  }
  if (tid < BM && q0 + tid < m) {
    long qi = q0 + tid;
#pragma unroll
    for (int i = 0; i < KMAX; i++) {
      if (i < kk) {
        out_ids[qi * kk + i] = li[i];
        out_sims[qi * kk + i] = li[i] == 0xFFFFFFFFu ? -INFINITY : ls[i];
      }
    }
  }
}

// Merge of the ranks' lists after the all-gather: per query, the best kk of
// world x kk candidates by (larger score, then lower id); the shards' ids are
// disjoint, and missing entries (0xFFFFFFFF) never enter.
__global__ void k_topk_merge(const uint32_t* __restrict__ stage, long m, int kk, int world,
                             uint32_t* __restrict__ out_ids, float* __restrict__ out_sims) {
  const long qi = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (qi >= m) return;
  float ls[KMAX];
  uint32_t li[KMAX];
#pragma unroll
  for (int i = 0; i < KMAX; i++) {
    ls[i] = -INFINITY;
    li[i] = 0xFFFFFFFFu;
  }
  const long per = 2 * m * (long)kk;  // words per rank: ids then sims
  for (int r = 0; r < world; r++) {
    const uint32_t* ids = stage + r * per;
    const float* sims = reinterpret_cast<const float*>(stage + r * per + m * (long)kk);
    for (int t = 0; t < kk; t++) {
      const uint32_t cj0 = ids[qi * kk + t];
      if (cj0 == 0xFFFFFFFFu) break;  // lists are best first: the rest are missing too
      float cv = sims[qi * kk + t];
      uint32_t cj = cj0;
#pragma unroll
      for (int i = 0; i < KMAX; i++) {
        const bool b = cv > ls[i] || (cv == ls[i] && cj < li[i]);
        const float tv = ls[i];
        const uint32_t tj = li[i];
        ls[i] = b ? cv : tv;
        li[i] = b ? cj : tj;
        cv = b ? tv : cv;
        cj = b ? tj : cj;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < KMAX; i++) {
    if (i < kk) {
      out_ids[qi * kk + i] = li[i];
      out_sims[qi * kk + i] = li[i] == 0xFFFFFFFFu ? -INFINITY : ls[i];
    }
  }
}

}  // namespace

void topk(eb_engine* e, const float* q, size_t m, const float* data, size_t n, size_t d,
          size_t kk, bool exclude_self, uint32_t* ids, float* sims, size_t id0,
          bool collective) {
  // A self-join (queries and data the same host rows) copies the rows once.
  const bool self_join = q == data && m == n;
  float* dq = e->scratch_get<float>("tk_q", m * d);
  float* dd = self_join ? dq : e->scratch_get<float>("tk_data", n * d);
  const bool group = collective && e->world > 1;
  // In a group the local lists land in this rank's share of the exchange
  // buffer (ids, then sims), which is all-gathered and merged.
  uint32_t* stage = group ? e->scratch_get<uint32_t>("tk_stage", (size_t)e->world * 2 * m * kk)
                          : nullptr;
  uint32_t* di = group ? stage + (size_t)e->rank * 2 * m * kk
                       : e->scratch_get<uint32_t>("tk_ids", m * kk);
  float* ds = group ? reinterpret_cast<float*>(di + m * kk) : e->scratch_get<float>("tk_sims", m * kk);
  h2d(e, dq, q, m * d * 4, e->stream);
  if (n && !self_join)
    h2d(e, dd, data, n * d * 4, e->stream);
  if (!topk_screen(e, dq, m, dd, n, d, kk, exclude_self, di, ds, id0)) {
    unsigned grid = (unsigned)((m + BM - 1) / BM);
    k_topk_exact<<<grid, NT, 0, e->stream>>>(dq, (long)m, dd, (long)n, (int)d, (int)kk,
                                             exclude_self ? 1 : 0, (long)id0, nullptr, (long)n, 0,
                                             di, ds);
    EB_LAUNCH("topk");
  }
  if (group) {
    group_allgather(e, stage, 2 * m * kk);
    di = e->scratch_get<uint32_t>("tk_ids", m * kk);
    ds = e->scratch_get<float>("tk_sims", m * kk);
    k_topk_merge<<<(unsigned)((m + 127) / 128), 128, 0, e->stream>>>(stage, (long)m, (int)kk,
                                                                     e->world, di, ds);
    EB_LAUNCH("topk merge");
  }
  d2h(e, ids, di, m * kk * 4, e->stream);
  d2h(e, sims, ds, m * kk * 4, e->stream);
  sync(e);
}

// Exact top-kk of L device-resident queries (global ids qids, for
// exclude_self) against n device-resident data rows: the data is split into
// up to one chunk per SM, every (64 queries, chunk) pair is a block, and the
// chunks' lists are merged; results (L x kk) stay on the device.
void topk_exact_device(eb_engine* e, const float* q, size_t L, const uint32_t* qids,
                       const float* data, size_t n, size_t d, size_t kk, bool exclude_self,
                       uint32_t* ids, float* sims, size_t id0) {
  if (L == 0) return;
  const size_t nch = std::max<size_t>(1, std::min<size_t>((size_t)e->num_sms, (n + 4095) / 4096));
  const size_t chunk = (n + nch - 1) / nch;
  const size_t per = 2 * L * kk;
  uint32_t* stage = e->scratch_get<uint32_t>("tk_chunks", nch * per);
  dim3 grid((unsigned)((L + BM - 1) / BM), (unsigned)nch);
  k_topk_exact<<<grid, NT, 0, e->stream>>>(q, (long)L, data, (long)n, (int)d, (int)kk,
                                           exclude_self ? 1 : 0, (long)id0, qids, (long)chunk,
                                           (long)per,
                                           stage, reinterpret_cast<float*>(stage + L * kk));
  EB_LAUNCH("topk chunks");
  k_topk_merge<<<(unsigned)((L + 127) / 128), 128, 0, e->stream>>>(stage, (long)L, (int)kk,
                                                                   (int)nch, ids, sims);
  EB_LAUNCH("topk chunk merge");
}

}  // namespace eb
