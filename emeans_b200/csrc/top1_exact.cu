// Exact FP32 top-1 on the SIMT pipes: every dot is one sequential FMA chain
// over the d columns, the float order of the reference CPU kernel
// (crates/emeans-core/src/assign/fused.rs:12-16). The running best keeps the
// lower id on ties (assign.rs:423-443); L2 keys are cnorm - 2 dot with one
// rounding and scores max(sum x^2 + key, 0) (assign.rs:497-502).
//
// This kernel serves the calls the tensor-core screen does not take (small
// problems, the exact mode). Tile: 64 rows x 64 centroids per block of 256
// threads (4x4 per thread), 16 columns of d per stage.
#include <cuda_runtime.h>

#include <climits>
#include <mutex>
#include <string>

#include "engine.h"

namespace eb {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

struct Best {
  float v;
  uint32_t j;
};

template <bool IP>
__device__ __forceinline__ bool better(float av, uint32_t aj, float bv, uint32_t bj) {
  return IP ? (av > bv || (av == bv && aj < bj)) : (av < bv || (av == bv && aj < bj));
}

template <bool IP>
__global__ void __launch_bounds__(NT) k_top1_exact(
    const float* __restrict__ x, long n, int d, const uint32_t* __restrict__ ids, long r0, long r1,
    const float* __restrict__ c, const float* __restrict__ cnorm, long k,
    const float* __restrict__ xnorm, int xnorm_by_row, uint32_t* __restrict__ labels,
    float* __restrict__ scores, uint32_t* status) {
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  __shared__ long pos_of[BM];
  __shared__ long row_of[BM];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const long total = r1 - r0;

  // Tiles of BM rows, grid-stride.
  for (long tile = blockIdx.x; tile * BM < total; tile += gridDim.x) {
  const long b0 = r0 + tile * BM;
  const long nrows = min((long)BM, r1 - b0);
  if (tid < BM) {
    long p = tid < nrows ? b0 + tid : -1;
    pos_of[tid] = p;
    long row = p < 0 ? 0 : (ids ? (long)ids[p] : p);
    if (row >= n) {
      atomicOr(status, ST_BAD_ROW);
      row = 0;
    }
    row_of[tid] = row;
  }
  __syncthreads();

  // Loader mapping: row (or centroid) lr = tid / 4, columns (tid % 4) * 4 .. +3.
  const int lr = tid >> 2, lc = (tid & 3) * 4;
  const float* arow = x + row_of[lr] * (long)d;
  const bool a_live = lr < nrows;
  const bool vec = (d & 3) == 0;

  float best_v[4];
  uint32_t best_j[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    best_v[i] = IP ? -INFINITY : INFINITY;
    best_j[i] = 0;
  }

  for (long n0 = 0; n0 < k; n0 += BN) {
    const long cj = n0 + lr;
    const float* brow = c + cj * (long)d;
    const bool b_live = cj < k;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < d; k0 += BK) {
      // Stage A and B columns k0..k0+BK (zeros past d; never used in the chain).
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
        for (int q = 0; q < 4; q++) {
          int t = k0 + lc + q;
          av[q] = (a_live && t < d) ? __ldg(arow + t) : 0.0f;
          bv[q] = (b_live && t < d) ? __ldg(brow + t) : 0.0f;
        }
      }
#pragma unroll
      for (int q = 0; q < 4; q++) {
        As[lc + q][lr] = av[q];
        Bs[lc + q][lr] = bv[q];
      }
      __syncthreads();
      const int kmax = min(BK, d - k0);
      if (kmax == BK) {
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
          float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
          float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
          float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
      } else {
        for (int kk = 0; kk < kmax; kk++) {
          float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
          float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
          float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
      }
      __syncthreads();
    }
    // Fold this tile into the running best, columns in increasing order.
#pragma unroll
    for (int j = 0; j < 4; j++) {
      long col = n0 + tx * 4 + j;
      if (col >= k) break;
      float cn = IP ? 0.0f : __ldg(cnorm + col);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float v = IP ? acc[i][j] : __fsub_rn(cn, __fmul_rn(2.0f, acc[i][j]));
        if (IP ? (v > best_v[i]) : (v < best_v[i])) {
          best_v[i] = v;
          best_j[i] = (uint32_t)col;
        }
      }
    }
  }

  // Merge the 16 threads of each row group (a half-warp), lower id on ties.
#pragma unroll
  for (int i = 0; i < 4; i++) {
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
      float ov = __shfl_xor_sync(0xFFFFFFFFu, best_v[i], off);
      uint32_t oj = __shfl_xor_sync(0xFFFFFFFFu, best_j[i], off);
      if (better<IP>(ov, oj, best_v[i], best_j[i])) {
        best_v[i] = ov;
        best_j[i] = oj;
      }
    }
  }
  if (tx == 0) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      int r = ty * 4 + i;
      if (r >= nrows) continue;
      long p = pos_of[r];
      float s = best_v[i];
      if (!IP) {
        float xn;
        if (xnorm) {
          xn = xnorm_by_row ? xnorm[row_of[r]] : xnorm[p - r0];
        } else {
          // Sequential sum of squares in the CPU order, for this row only.
          const float* xr = x + row_of[r] * (long)d;
          xn = -0.0f;
          for (int t = 0; t < d; t++) {
            const float v = __ldg(xr + t);
            xn = __fadd_rn(xn, __fmul_rn(v, v));
          }
        }
        s = fmaxf(__fadd_rn(xn, s), 0.0f);
      }
      labels[p] = best_j[i];
      scores[p] = s;
    }
  }
  __syncthreads();  // pos_of / row_of are rewritten by the next tile
  }
}

}  // namespace

void top1_exact(eb_engine* e, const Top1Args& a) {
  const size_t rows = a.r1 - a.r0;
  if (rows == 0) return;
  const float* xn = nullptr;
  int by_row = 0;
  if (a.metric == EB_L2) {
    if (a.xnorm) {
      xn = a.xnorm;
      by_row = 1;
    } else {
      float* t = e->scratch_get<float>("top1_xnorm", a.r1 - a.r0);
      sel_row_norms(e, a.x, a.n, a.d, a.ids, a.r0, a.r1, t);
      xn = t;
    }
  }
  const unsigned grid = (unsigned)((rows + BM - 1) / BM);
  if (a.metric == EB_IP)
    k_top1_exact<true><<<grid, NT, 0, e->stream>>>(a.x, (long)a.n, (int)a.d, a.ids, (long)a.r0,
                                                   (long)a.r1, a.c, a.cnorm,
                                                   (long)a.k, xn, by_row, a.labels, a.scores,
                                                   e->d_status);
  else
    k_top1_exact<false><<<grid, NT, 0, e->stream>>>(a.x, (long)a.n, (int)a.d, a.ids, (long)a.r0,
                                                    (long)a.r1, a.c, a.cnorm,
                                                    (long)a.k, xn, by_row, a.labels, a.scores,
                                                    e->d_status);
  EB_LAUNCH("top1_exact");
  e->stats.exact_rows += rows;
}

// ---------------------------------------------------------------- no-alloc entry
//
// eb_top1_exact_noalloc runs the kernel above for callers that may not
// allocate device memory while a call is in progress: a serving process that
// reserves its device memory once at start-up and must keep its footprint
// fixed per request, or a caller on a latency budget that cannot take the
// pause (or the failure) a pool allocation may bring under memory pressure.
// The engine's top-1 keeps its L2 row norms in grow-only scratch, which can
// allocate on a larger call; this entry keeps them in the fixed device array
// below instead, so the call itself allocates nothing.
//
// The first call on a device does the set-up (looking up this device's copy
// of the array, which may load the module): make it before any stream
// capture. The array is one per device and shared by every engine on it, so
// two calls in flight at once on one device (different streams or engines)
// race on it; calls on one stream are ordered and safe. Nothing in it needs
// to start at zero: every norm a call reads is written earlier in that call.
namespace {

constexpr size_t kNoAllocRows = EB_NOALLOC_MAX_ROWS;  // 4 MiB of row norms
static __device__ __align__(256) float g_noalloc_xnorm[kNoAllocRows];

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_addr[kNoAllocDevices] = {};

// This device's copy of the array; the caller has made the device current.
float* noalloc_scratch(int device) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (device < 0 || device >= kNoAllocDevices)
    throw Error(EB_ERROR, "device ordinal out of range for the no-alloc scratch");
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_xnorm);
    if (rc != cudaSuccess || p == nullptr)
      throw Error(EB_ERROR, std::string("cudaGetSymbolAddress(no-alloc scratch): ") +
                                cudaGetErrorString(rc));
    g_noalloc_addr[device] = static_cast<float*>(p);
  }
  return g_noalloc_addr[device];
}

struct CurrentDevice {
  int prev = -1;
  explicit CurrentDevice(int device) {
    cudaGetDevice(&prev);
    if (prev != device) EB_CUDA(cudaSetDevice(device));
  }
  ~CurrentDevice() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

}  // namespace eb

extern "C" int eb_top1_exact_noalloc(eb_engine* e, const float* x, size_t n, size_t d,
                                     const uint32_t* ids, size_t r0, size_t r1, const float* c,
                                     const float* cnorm, size_t k, int metric, uint32_t* labels,
                                     float* scores) {
  using namespace eb;
  try {
    ensure(e != nullptr, "engine is null");
    ensure(x && c && labels && scores, "a device pointer is null");
    ensure(d > 0, "d must be positive");
    // The kernel indexes columns with int and rows with long.
    ensure(d <= (size_t)INT_MAX, "d must be at most 2^31 - 1");
    ensure(n <= (size_t)LONG_MAX / d, "n * d overflows");
    ensure(k <= (size_t)LONG_MAX / d, "k * d overflows");
    ensure(metric == EB_L2 || metric == EB_IP, "unknown metric");
    ensure(r0 <= r1, "bad row range");
    if (!ids) ensure(r1 <= n, "row range past the data");
    ensure(k > 0 && k <= 0xFFFFFFFFull, "k must be in 1 .. 2^32 - 1");
    if (metric == EB_L2) ensure(cnorm != nullptr, "L2 needs centroid norms");
    ensure(r1 - r0 <= kNoAllocRows,
           "the no-alloc top-1 takes at most " + std::to_string(kNoAllocRows) +
               " rows per call (got " + std::to_string(r1 - r0) + ")");
    CurrentDevice dev(e->device);
    float* xn = noalloc_scratch(e->device);
    const size_t rows = r1 - r0;
    if (rows > 0) {
      if (metric == EB_L2) sel_row_norms(e, x, n, d, ids, r0, r1, xn);
      const unsigned grid = (unsigned)((rows + BM - 1) / BM);
      if (metric == EB_IP)
        k_top1_exact<true><<<grid, NT, 0, e->stream>>>(x, (long)n, (int)d, ids, (long)r0,
                                                       (long)r1, c, cnorm, (long)k, nullptr, 0,
                                                       labels, scores, e->d_status);
      else
        k_top1_exact<false><<<grid, NT, 0, e->stream>>>(x, (long)n, (int)d, ids, (long)r0,
                                                        (long)r1, c, cnorm, (long)k, xn, 0,
                                                        labels, scores, e->d_status);
      EB_LAUNCH("top1_exact_noalloc");
      e->stats.exact_rows += rows;
    }
    set_last_error("");
    return EB_OK;
  } catch (const Error& err) {
    set_last_error(err.what());
    return err.code;
  } catch (const std::exception& err) {
    set_last_error(std::string("internal: ") + err.what());
    return EB_INTERNAL;
  }
}
