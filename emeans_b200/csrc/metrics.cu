// Internal quality scores of a labelling (crates/emeans-cluster/src/metrics.rs:
// 115-274) on the device: cosine silhouette, Calinski-Harabasz,
// Davies-Bouldin and the spherical objective of unit rows.
//
// The reference forms the cluster sums in f64 in row order, takes one n x k_eff
// product of the rows with the f32-rounded sums (gemm_nt, crates/emeans-core/
// src/assign.rs:813-825, in row blocks) and scores every row from its row of
// that product. Here:
//  - k_sum64: the f64 sums, one thread per (cluster, column), the cluster's
//    rows in row order (the stable sort by label of the scatter-add);
//  - k_cluster_prep: f32 sums, sum of squares and size of the live clusters;
//  - k_silhouette: the product as FP32 FMA chains in 128 x 128 tiles, and in its
//    epilogue each row's own-cluster product and the best other cluster's
//    product / size, so that the n x k_eff matrix never reaches memory; the
//    row's silhouette, objective term and distance to its cluster mean are
//    written in f64 with the reference's operation order (no contraction);
//  - k_db: Davies-Bouldin's worst ratio per cluster over the cluster means.
// The host adds the per-row terms in row order and forms Calinski-Harabasz as
// metrics.rs:189-216 does.
#include <cuda_runtime.h>

#include <cmath>
#include <vector>

#include "engine.h"

namespace eb {
namespace {

unsigned nblocks(size_t n, unsigned per) { return (unsigned)((n + per - 1) / per); }

// sums[j][t] = sum of (double)x[row][t] over the rows of cluster j in row
// order, from +0 (metrics.rs:127-134).
constexpr uint32_t kStage = 1024;
// Block b takes the b / cb-th largest cluster (by_size) and its column block
// b % cb, so that the longest chains start first.
__global__ void __launch_bounds__(128) k_sum64(const float* __restrict__ x, int d, int cb,
                                               const uint32_t* __restrict__ order,
                                               const uint32_t* __restrict__ start,
                                               const uint32_t* __restrict__ by_size,
                                               double* __restrict__ sums) {
  pdl_wait();
  __shared__ uint32_t ord_s[kStage];
  const long j = by_size[blockIdx.x / cb];
  const int t = (blockIdx.x % cb) * blockDim.x + threadIdx.x;
  const bool active = t < d;
  const float* xt = x + (active ? t : 0);
  const uint32_t b = start[j], en = start[j + 1];
  double s = 0.0;
  for (uint32_t c0 = b; c0 < en; c0 += kStage) {
    const uint32_t m = min(en - c0, kStage);
    __syncthreads();  // the previous chunk's ids are no longer read
    for (uint32_t u = threadIdx.x; u < m; u += blockDim.x) ord_s[u] = order[c0 + u];
    __syncthreads();
    if (!active) continue;
    uint32_t i = 0;
    for (; i + 16 <= m; i += 16) {
      float v[16];
#pragma unroll
      for (int q = 0; q < 16; q++) v[q] = __ldg(xt + (long)ord_s[i + q] * d);
#pragma unroll
      for (int q = 0; q < 16; q++) s = __dadd_rn(s, (double)v[q]);
    }
    for (; i < m; i++) s = __dadd_rn(s, (double)__ldg(xt + (long)ord_s[i] * d));
  }
  if (active) sums[j * d + t] = s;
}

// For live cluster s (label live[s]): c32 = (float)sums, sq = sequential sum
// of sums^2 (metrics.rs:141-148), size = its count, and its f64 mean
// sums / size (metrics.rs:218-227), stored column-major (meanT[t][s]) for
// k_db. One block per live cluster.
__global__ void k_cluster_prep(const double* __restrict__ sums, const uint32_t* __restrict__ live,
                               const uint32_t* __restrict__ counts, int d, long keff,
                               float* __restrict__ c32, double* __restrict__ sq,
                               double* __restrict__ size, double* __restrict__ meanT,
                               float* __restrict__ inv) {
  pdl_wait();
  const long s = blockIdx.x;
  const long j = live[s];
  const double nj = (double)counts[j];
  const double* row = sums + j * d;
  for (int t = threadIdx.x; t < d; t += blockDim.x) {
    const double v = row[t];
    c32[s * d + t] = (float)v;
    meanT[(long)t * keff + s] = __ddiv_rn(v, nj);
  }
  if (threadIdx.x == 0) {
    double a = -0.0;
    for (int t = 0; t < d; t++) a = __dadd_rn(a, __dmul_rn(row[t], row[t]));
    sq[s] = a;
    size[s] = nj;
    inv[s] = 1.0f / (float)nj;  // the tensor-core product's column weight
  }
}

// The per-row terms with the tensor-core product (screen_products), which
// picks each row's best other cluster b (the largest x_i . c32_s / n_s over
// s != o). Both products the row needs, x_i . c32_o and x_i . c32_b, are FP32
// FMA chains in column order, the SIMT kernel's values bit for bit (the
// distance and the silhouette's a cancel the own product against the row's
// norm, and the tensor cores' FP32 accumulation leans toward zero), so the
// scores equal the SIMT path's except where two clusters tie within the
// screen's rounding. Then the row's f64 sum of squares in column order and
// the same formulas as k_silhouette's epilogue. One warp per 32 rows: each
// 32-column slice of the warp's rows is read coalesced (a row per load, a
// column per lane) into shared memory, and each lane runs its own row's
// chains.
__global__ void __launch_bounds__(128) k_row_terms(
    const float* __restrict__ x, long n, int d, const uint32_t* __restrict__ labels,
    const uint32_t* __restrict__ slot, const float* __restrict__ c32,
    const uint32_t* __restrict__ best, const double* __restrict__ size,
    const double* __restrict__ sq, long keff, double* __restrict__ sil, double* __restrict__ obj,
    double* __restrict__ dist, double* __restrict__ xx_out) {
  pdl_wait();
  __shared__ float tile[4][32][33];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long r0 = ((long)blockIdx.x * 4 + w) * 32;
  if (r0 >= n) return;
  float(*t)[33] = tile[w];
  const long myrow = min(r0 + lane, n - 1);
  const float* crow = c32 + (long)slot[labels[myrow]] * d;
  const uint32_t bcol = best[myrow];
  const bool has_b = bcol < (uint32_t)keff;
  const float* brow = c32 + (long)(has_b ? bcol : 0) * d;
  double xv = -0.0;
  float gf = 0.0f, gb = 0.0f;
  // Each lane reads its two centroid rows' slice as eight 16-byte loads
  // each (a whole 128-byte line) when the rows allow it.
  const bool vec = (d & 3) == 0 && ((uintptr_t)c32 & 15) == 0;
  for (int c0 = 0; c0 < d; c0 += 32) {
    {
      float v[32];
#pragma unroll
      for (int r = 0; r < 32; r++) {
        const long row = r0 + r;
        v[r] = (row < n && c0 + lane < d) ? __ldg(x + row * d + c0 + lane) : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < 32; r++) t[r][lane] = v[r];
    }
    __syncwarp();
    const int cmax = min(32, d - c0);
    if (vec && cmax == 32) {
      float cv[32], bv[32];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(crow + c0) + q);
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(brow + c0) + q);
        cv[4 * q] = a4.x; cv[4 * q + 1] = a4.y; cv[4 * q + 2] = a4.z; cv[4 * q + 3] = a4.w;
        bv[4 * q] = b4.x; bv[4 * q + 1] = b4.y; bv[4 * q + 2] = b4.z; bv[4 * q + 3] = b4.w;
      }
#pragma unroll
      for (int c = 0; c < 32; c++) {
        const float a = t[lane][c];
        const double q = (double)a;
        xv = __dadd_rn(xv, __dmul_rn(q, q));
        gf = __fmaf_rn(a, cv[c], gf);
        gb = __fmaf_rn(a, bv[c], gb);
      }
    } else {
      for (int c = 0; c < cmax; c++) {
        const float a = t[lane][c];
        const double q = (double)a;
        xv = __dadd_rn(xv, __dmul_rn(q, q));
        gf = __fmaf_rn(a, __ldg(crow + c0 + c), gf);
        gb = __fmaf_rn(a, __ldg(brow + c0 + c), gb);
      }
    }
    __syncwarp();
  }
  const long row = r0 + lane;
  if (row >= n) return;
  const uint32_t o = slot[labels[row]];
  const double na = size[o], sqo = sq[o];
  const double g = (double)gf;
  const double t1 = __ddiv_rn(__dmul_rn(2.0, g), na);
  const double t2 = __ddiv_rn(sqo, __dmul_rn(na, na));
  dist[row] = __dsqrt_rn(fmax(__dadd_rn(__dsub_rn(xv, t1), t2), 0.0));
  const double cosc = __ddiv_rn(g, fmax(__dsqrt_rn(sqo), 1e-30));
  obj[row] = __dsub_rn(2.0, __dmul_rn(2.0, cosc));
  double sv = 0.0;
  if (keff >= 2 && na >= 2.0) {
    const double a = __dsub_rn(1.0, __ddiv_rn(__dsub_rn(g, xv), __dsub_rn(na, 1.0)));
    const double vm = has_b ? __ddiv_rn((double)gb, size[bcol])
                            : (bcol == 0xFFFFFFFFu ? -INFINITY : NAN);
    const double bb = __dsub_rn(1.0, vm);
    const double m = fmax(a, bb);
    sv = m > 0.0 ? __ddiv_rn(__dsub_rn(bb, a), m) : 0.0;
  }
  sil[row] = sv;
  xx_out[row] = xv;
}

// Per row i with live cluster o = slot[labels[i]] (metrics.rs:160-185):
//   g_s  = x_i . c32_s (FP32 FMA chain over the columns)
//   xx   = sequential sum of x^2 in f64
//   dist = sqrt(max(xx - 2 g_o / n_o + sq_o / n_o^2, 0))
//   obj  = 2 - 2 g_o / max(sqrt(sq_o), 1e-30)
//   sil  = (b - a) / max(a, b) with a = 1 - (g_o - xx) / (n_o - 1) and
//          b = min over s != o of 1 - g_s / n_s (= 1 - max of g_s / n_s: the
//          rounding of 1 - q is monotone), 0 when k_eff < 2 or n_o < 2.
// Tile: 128 rows x 128 clusters per block of 256 threads, 8 x 8 per thread
// (rows ty*4 + {0..3} and 64 + ty*4 + {0..3}, clusters likewise by tx), so
// that four 16-byte shared-memory reads feed 64 FMAs; 8 columns per stage;
// rows in tiles, grid-stride.
constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

__device__ __forceinline__ int half_idx(int base, int q) { return (q < 4 ? 0 : 64) + base + (q & 3); }

__global__ void __launch_bounds__(NT) k_silhouette(
    const float* __restrict__ x, long n, int d, const uint32_t* __restrict__ labels,
    const uint32_t* __restrict__ slot, const float* __restrict__ c32,
    const double* __restrict__ size, const double* __restrict__ sq, long keff,
    double* __restrict__ sil, double* __restrict__ obj, double* __restrict__ dist,
    double* __restrict__ xx_out) {
  pdl_wait();
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  __shared__ int own_of[BM];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int lr = tid >> 1, lc = (tid & 1) * 4;  // loader: row (cluster) lr, columns lc..lc+3
  const bool vec = (d & 3) == 0;

  for (long tile = blockIdx.x; tile * BM < n; tile += gridDim.x) {
    const long b0 = tile * BM;
    const long nrows = min((long)BM, n - b0);
    if (tid < BM) own_of[tid] = tid < nrows ? (int)slot[labels[b0 + tid]] : 0;
    __syncthreads();
    const float* arow = x + (b0 + min((long)lr, nrows - 1)) * (long)d;
    const bool a_live = lr < nrows;

    int own[8];
    double vmax[8], xxr[8];
    float dot[8];
    bool have[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      own[i] = own_of[half_idx(ty * 4, i)];
      vmax[i] = -INFINITY;
      xxr[i] = -0.0;
      dot[i] = 0.0f;
      have[i] = false;
    }

    for (long n0 = 0; n0 < keff; n0 += BN) {
      const long cj = n0 + lr;
      const bool b_live = cj < keff;
      const float* brow = c32 + (b_live ? cj : 0) * (long)d;
      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

      // Stage k0's columns lc..lc+3 of the loader's row and cluster (zeros
      // past d; never used in the chain).
      auto load = [&](int k0, float* av, float* bv) {
        if (vec && k0 + lc + 4 <= d) {
          const float4 a4 = a_live ? __ldg(reinterpret_cast<const float4*>(arow + k0 + lc))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 b4 = b_live ? __ldg(reinterpret_cast<const float4*>(brow + k0 + lc))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
          av[0] = a4.x; av[1] = a4.y; av[2] = a4.z; av[3] = a4.w;
          bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
        } else {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int t = k0 + lc + q;
            av[q] = (a_live && t < d) ? __ldg(arow + t) : 0.0f;
            bv[q] = (b_live && t < d) ? __ldg(brow + t) : 0.0f;
          }
        }
      };
      float av[4], bv[4];
      load(0, av, bv);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        As[lc + q][lr] = av[q];
        Bs[lc + q][lr] = bv[q];
      }
      __syncthreads();
      for (int k0 = 0; k0 < d; k0 += BK) {
        // The next stage's loads are in flight while this stage is computed.
        const bool more = k0 + BK < d;
        if (more) load(k0 + BK, av, bv);
        const int kmax = min(BK, d - k0);
        if (n0 == 0 && tx == 0) {
          // The rows' sums of squares, once per tile, in column order.
          for (int kk = 0; kk < kmax; kk++)
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const double v = (double)As[kk][half_idx(ty * 4, i)];
              xxr[i] = __dadd_rn(xxr[i], __dmul_rn(v, v));
            }
        }
        auto step = [&](int kk) {
          const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
          const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][64 + ty * 4]);
          const float4 b0v = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
          const float4 b1v = *reinterpret_cast<const float4*>(&Bs[kk][64 + tx * 4]);
          const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const float b[8] = {b0v.x, b0v.y, b0v.z, b0v.w, b1v.x, b1v.y, b1v.z, b1v.w};
#pragma unroll
          for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        };
        if (kmax == BK) {
#pragma unroll
          for (int kk = 0; kk < BK; kk++) step(kk);
        } else {
          for (int kk = 0; kk < kmax; kk++) step(kk);
        }
        __syncthreads();  // every thread is done with this stage
        if (more) {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            As[lc + q][lr] = av[q];
            Bs[lc + q][lr] = bv[q];
          }
        }
        __syncthreads();
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const long col = n0 + half_idx(tx * 4, j);
        if (col >= keff) continue;
        const double nc = __ldg(size + col);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          if (col == own[i]) {
            dot[i] = acc[i][j];
            have[i] = true;
          } else {
            vmax[i] = fmax(vmax[i], __ddiv_rn((double)acc[i][j], nc));
          }
        }
      }
    }

    // Merge the 16 threads of each row group (a half-warp).
#pragma unroll
    for (int i = 0; i < 8; i++) {
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) {
        const double ov = __shfl_xor_sync(0xFFFFFFFFu, vmax[i], off);
        const float od = __shfl_xor_sync(0xFFFFFFFFu, dot[i], off);
        const int oh = __shfl_xor_sync(0xFFFFFFFFu, (int)have[i], off);
        vmax[i] = fmax(vmax[i], ov);
        if (!have[i] && oh) {
          dot[i] = od;
          have[i] = true;
        }
      }
    }
    if (tx == 0) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int r = half_idx(ty * 4, i);
        if (r >= nrows) continue;
        const long row = b0 + r;
        const int o = own[i];
        const double na = size[o], sqo = sq[o];
        const double g = (double)dot[i], xv = xxr[i];
        const double t1 = __ddiv_rn(__dmul_rn(2.0, g), na);
        const double t2 = __ddiv_rn(sqo, __dmul_rn(na, na));
        dist[row] = __dsqrt_rn(fmax(__dadd_rn(__dsub_rn(xv, t1), t2), 0.0));
        const double cosc = __ddiv_rn(g, fmax(__dsqrt_rn(sqo), 1e-30));
        obj[row] = __dsub_rn(2.0, __dmul_rn(2.0, cosc));
        double sv = 0.0;
        if (keff >= 2 && na >= 2.0) {
          const double a = __dsub_rn(1.0, __ddiv_rn(__dsub_rn(g, xv), __dsub_rn(na, 1.0)));
          const double bb = __dsub_rn(1.0, vmax[i]);
          const double m = fmax(a, bb);
          sv = m > 0.0 ? __ddiv_rn(__dsub_rn(bb, a), m) : 0.0;
        }
        sil[row] = sv;
        xx_out[row] = xv;
      }
    }
    __syncthreads();  // own_of is rewritten by the next tile
  }
}

// worst[a] = max over b != a of (spread_a + spread_b) / |mean_a - mean_b|
// (infinite for equal means), folded from 0 (metrics.rs:233-256); each
// distance is a sequential f64 chain over the columns. The chain of (a, b)
// and the one of (b, a) are the same bits ((ma - mb)^2 = (mb - ma)^2, and the
// spreads' sum commutes), so each pair is computed once, for b > a, and
// folded into both worst[a] and worst[b]. A block takes kDbA clusters a
// (their 32-column slices staged in shared memory) and 256 clusters b (one
// per thread, the means column-major so that a warp's 32 b's at one column
// are one coalesced read), with kDbA chains per thread; blocks wholly below
// the diagonal do nothing. The maxima are non-negative doubles (or +inf),
// whose bit patterns order like their values: atomic maxima on the bits, into
// worst zeroed by the caller.
constexpr int kDbA = 16, kDbB = 256, kDbT = 32;
__device__ __forceinline__ void atomic_max_nonneg(double* p, double v) {
  atomicMax(reinterpret_cast<unsigned long long*>(p), (unsigned long long)__double_as_longlong(v));
}
__global__ void __launch_bounds__(kDbB) k_db(const double* __restrict__ meanT,
                                             const double* __restrict__ spread, long keff, int d,
                                             double* __restrict__ worst) {
  pdl_wait();
  __shared__ double as[kDbT][kDbA];
  __shared__ double red[kDbB / 32][kDbA];
  const long a0 = (long)blockIdx.y * kDbA;
  const long b = (long)blockIdx.x * kDbB + threadIdx.x;
  if ((long)blockIdx.x * kDbB + kDbB - 1 <= a0) return;  // every b <= every a: nothing here
  const long bc = min(b, keff - 1);
  double s[kDbA];
#pragma unroll
  for (int q = 0; q < kDbA; q++) s[q] = -0.0;
  for (int t0 = 0; t0 < d; t0 += kDbT) {
    const int tn = min(kDbT, d - t0);
    __syncthreads();  // the last slice is no longer read
    for (int u = threadIdx.x; u < kDbT * kDbA; u += kDbB) {
      const int tt = u / kDbA, q = u % kDbA;
      as[tt][q] = tt < tn ? __ldg(meanT + (long)(t0 + tt) * keff + min(a0 + q, keff - 1)) : 0.0;
    }
    __syncthreads();
    const double* col = meanT + (long)t0 * keff + bc;
    if (tn == kDbT) {
#pragma unroll 8
      for (int tt = 0; tt < kDbT; tt++) {
        const double mb = __ldg(col + (long)tt * keff);
#pragma unroll
        for (int q = 0; q < kDbA; q++) {
          const double df = __dsub_rn(as[tt][q], mb);
          s[q] = __dadd_rn(s[q], __dmul_rn(df, df));
        }
      }
    } else {
      for (int tt = 0; tt < tn; tt++) {
        const double mb = __ldg(col + (long)tt * keff);
#pragma unroll
        for (int q = 0; q < kDbA; q++) {
          const double df = __dsub_rn(as[tt][q], mb);
          s[q] = __dadd_rn(s[q], __dmul_rn(df, df));
        }
      }
    }
  }
  const bool bl = b < keff;
  const double sb = bl ? spread[b] : 0.0;
  double wb = 0.0;  // this b's maximum over the block's a's
  double wa[kDbA];
#pragma unroll
  for (int q = 0; q < kDbA; q++) {
    const long a = a0 + q;
    wa[q] = 0.0;
    if (!bl || a >= keff || b <= a) continue;
    const double m = __dsqrt_rn(s[q]);
    const double v = m > 0.0 ? __ddiv_rn(__dadd_rn(spread[a], sb), m) : INFINITY;
    wa[q] = v;
    wb = fmax(wb, v);
  }
  if (bl && wb > 0.0) atomic_max_nonneg(worst + b, wb);
  // Each a's maximum over the block's b's: warp shuffles, then across warps.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < kDbA; q++) {
    double v = wa[q];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmax(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    if (lane == 0) red[warp][q] = v;
  }
  __syncthreads();
  if (threadIdx.x < kDbA && a0 + threadIdx.x < keff) {
    double v = 0.0;
#pragma unroll
    for (int w = 0; w < kDbB / 32; w++) v = fmax(v, red[w][threadIdx.x]);
    if (v > 0.0) atomic_max_nonneg(worst + a0 + threadIdx.x, v);
  }
}

// grand[t] = sum over the live clusters, in label order, of sums[j][t] from
// +0 (metrics.rs:204-209). One thread per column.
__global__ void k_grand(const double* __restrict__ sums, const uint32_t* __restrict__ live,
                        long keff, int d, double* __restrict__ grand) {
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d) return;
  // One sequential chain per column; sixteen loads in flight ahead of it.
  double g = 0.0;
  long s = 0;
  for (; s + 16 <= keff; s += 16) {
    double v[16];
#pragma unroll
    for (int q = 0; q < 16; q++) v[q] = __ldg(sums + (long)live[s + q] * d + t);
#pragma unroll
    for (int q = 0; q < 16; q++) g = __dadd_rn(g, v[q]);
  }
  for (; s < keff; s++) g = __dadd_rn(g, sums[(long)live[s] * d + t]);
  grand[t] = g;
}

// Device memory for one call, released on the engine's stream.
struct Tmp {
  eb_engine* e;
  void* p = nullptr;
  Tmp(eb_engine* eng, size_t bytes) : e(eng) {
    EB_CUDA(cudaMallocAsync(&p, std::max<size_t>(bytes, 16), e->stream));
    e->device_allocs++;
  }
  ~Tmp() {
    if (p) cudaFreeAsync(p, e->stream);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

}  // namespace

void internal_scores(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* labels,
                     size_t k, eb_internal* out, uint64_t* sizes) {
  *out = eb_internal{};
  if (sizes)
    for (size_t j = 0; j < k; j++) sizes[j] = 0;
  if (n == 0) return;  // no clusters: every score 0 (metrics.rs:258-273 with n = 0)

  // Rows on the device: bound data in place, else one copy for this call.
  const bool reuse = e->bound && e->bound_host == x && e->bound_n == n && e->bound->d == d;
  std::unique_ptr<Tmp> xcopy;
  const float* xd;
  if (reuse) {
    xd = static_cast<const float*>(e->bound->ptr);
  } else {
    xcopy.reset(new Tmp(e, n * d * 4));
    h2d(e, xcopy->p, x, n * d * 4, e->stream);
    xd = xcopy->as<float>();
  }
  Tmp lab(e, n * 4), cnt(e, k * 4), sums(e, k * d * 8);
  h2d(e, lab.p, labels, n * 4, e->stream);
  const uint32_t *order, *start, *by_size;
  label_order(e, nullptr, 0, n, n, lab.as<uint32_t>(), k, cnt.as<uint32_t>(), &order, &start,
              &by_size);
  const unsigned cb = nblocks(d, 128);
  launch_pdl(e, k_sum64, (unsigned)(k * cb), 128, 0, xd, (int)d, (int)cb, order, start, by_size,
             sums.as<double>());
  EB_LAUNCH("metrics sums");

  std::vector<uint32_t> counts(k);
  d2h(e, counts.data(), cnt.p, k * 4, e->stream);
  sync(e);
  std::vector<uint32_t> live, slot(k, 0);
  for (size_t j = 0; j < k; j++) {
    if (sizes) sizes[j] = counts[j];
    if (counts[j] > 0) {
      slot[j] = (uint32_t)live.size();
      live.push_back((uint32_t)j);
    }
  }
  const size_t keff = live.size();
  Tmp dlive(e, keff * 4), dslot(e, k * 4), c32(e, keff * d * 4), sq(e, keff * 8),
      size(e, keff * 8), mean(e, keff * d * 8), inv(e, keff * 4);
  h2d(e, dlive.p, live.data(), keff * 4, e->stream);
  h2d(e, dslot.p, slot.data(), k * 4, e->stream);
  launch_pdl(e, k_cluster_prep, (unsigned)keff, 128, 0, sums.as<double>(), dlive.as<uint32_t>(),
             cnt.as<uint32_t>(), (int)d, (long)keff, c32.as<float>(), sq.as<double>(),
             size.as<double>(), mean.as<double>(), inv.as<float>());
  EB_LAUNCH("metrics cluster prep");

  Tmp sil(e, n * 8), obj(e, n * 8), dist(e, n * 8), xx(e, n * 8);
  // The n x k_eff product: on the tensor cores (the screen's split FP16
  // products in product mode) for calls large enough to pay, or always in
  // screen mode 2; FP32 FMA chains on the SIMT cores otherwise.
  const bool tensor = e->screen_mode == 2 ||
                      (e->screen_mode == 1 && n >= 4096 && keff >= 64 && d >= 16 && d <= 16384);
  if (tensor) {
    Tmp best(e, n * 4);
    screen_products(e, xd, n, d, reuse ? e->bound : nullptr, lab.as<uint32_t>(),
                    dslot.as<uint32_t>(), c32.as<float>(), inv.as<float>(), keff,
                    best.as<uint32_t>());
    launch_pdl(e, k_row_terms, nblocks(n, 128), 128, 0, xd, (long)n, (int)d, lab.as<uint32_t>(),
               dslot.as<uint32_t>(), c32.as<float>(), best.as<uint32_t>(), size.as<double>(),
               sq.as<double>(), (long)keff, sil.as<double>(), obj.as<double>(),
               dist.as<double>(), xx.as<double>());
    EB_LAUNCH("metrics row terms");
  } else {
    const unsigned tiles = nblocks(n, BM);
    const unsigned grid = std::min<unsigned>(tiles, (unsigned)e->num_sms * 4);
    launch_pdl(e, k_silhouette, grid, NT, 0, xd, (long)n, (int)d, lab.as<uint32_t>(),
               dslot.as<uint32_t>(), c32.as<float>(), size.as<double>(), sq.as<double>(),
               (long)keff, sil.as<double>(), obj.as<double>(), dist.as<double>(), xx.as<double>());
    EB_LAUNCH("metrics silhouette");
  }

  Tmp grand_d(e, d * 8);
  launch_pdl(e, k_grand, nblocks(d, 128), 128, 0, sums.as<double>(), dlive.as<uint32_t>(),
             (long)keff, (int)d, grand_d.as<double>());
  EB_LAUNCH("metrics grand");

  // Read-back into the engine's pinned buffers (one DMA each, no staging).
  double* h_sil = e->pinned_get<double>("met_sil", n);
  double* h_obj = e->pinned_get<double>("met_obj", n);
  double* h_dist = e->pinned_get<double>("met_dist", n);
  double* h_xx = e->pinned_get<double>("met_xx", n);
  double* h_grand = e->pinned_get<double>("met_grand", d);
  double* h_sq = e->pinned_get<double>("met_sq", keff);
  EB_CUDA(cudaMemcpyAsync(h_sil, sil.p, n * 8, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(h_obj, obj.p, n * 8, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(h_dist, dist.p, n * 8, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(h_xx, xx.p, n * 8, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(h_grand, grand_d.p, d * 8, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(h_sq, sq.p, keff * 8, cudaMemcpyDeviceToHost, e->stream));
  sync(e);

  // Row-order sums (metrics.rs:178-184).
  double sil_sum = 0.0, obj_sum = 0.0;
  std::vector<double> scatter(keff, 0.0);
  for (size_t i = 0; i < n; i++) {
    sil_sum += h_sil[i];
    obj_sum += h_obj[i];
    scatter[slot[labels[i]]] += h_dist[i];
  }
  const double nf = (double)n;

  // Calinski-Harabasz (metrics.rs:189-216).
  double total_xx = -0.0;
  for (size_t i = 0; i < n; i++) total_xx += h_xx[i];
  double wsum = -0.0;
  for (size_t s = 0; s < keff; s++) wsum += h_sq[s] / (double)counts[live[s]];
  const double within = total_xx - wsum;
  double gsq = -0.0;
  for (size_t t = 0; t < d; t++) gsq += h_grand[t] * h_grand[t];
  const double total = total_xx - gsq / nf;
  const double between = total - within;
  double ch = 0.0;
  if (!(keff < 2 || n <= keff || within <= 0.0))
    ch = (between / (double)(keff - 1)) / (within / (double)(n - keff));

  // Davies-Bouldin (metrics.rs:217-256).
  double db = 0.0;
  if (keff >= 2) {
    std::vector<double> spread(keff);
    for (size_t s = 0; s < keff; s++) spread[s] = scatter[s] / (double)counts[live[s]];
    Tmp dspread(e, keff * 8), dworst(e, keff * 8);
    h2d(e, dspread.p, spread.data(), keff * 8, e->stream);
    EB_CUDA(cudaMemsetAsync(dworst.p, 0, keff * 8, e->stream));
    launch_pdl(e, k_db, dim3(nblocks(keff, kDbB), nblocks(keff, kDbA)), kDbB, 0,
               mean.as<double>(), dspread.as<double>(), (long)keff, (int)d, dworst.as<double>());
    EB_LAUNCH("metrics davies-bouldin");
    std::vector<double> worst(keff);
    d2h(e, worst.data(), dworst.p, keff * 8, e->stream);
    sync(e);
    double acc = -0.0;
    for (size_t s = 0; s < keff; s++) acc += worst[s];
    db = acc / (double)keff;
  }

  out->k_eff = keff;
  out->silhouette = sil_sum / nf;
  out->calinski_harabasz = ch;
  out->davies_bouldin = db;
  out->objective = obj_sum / nf;
}

}  // namespace eb
