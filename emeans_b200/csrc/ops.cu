// The update ops of the hot path: row norms, normalisation, the EMA step,
// revival splits and the deterministic scatter-add. Each is bit-equal to the
// reference CPU float order (crates/emeans-core/src/core/cpu.rs): every
// rounding is spelled with an explicit __f*_rn intrinsic, so no FMA
// contraction can change a bit, and sums run in the reference's order.
#include <cuda_runtime.h>

#include "engine.h"

namespace eb {
namespace {

constexpr int kRowThreads = 64;

// Sequential sum of rounded squares of one row, in column order
// (assign.rs:150-155: `r.iter().map(|v| v * v).sum()`).
__device__ __forceinline__ float row_sumsq(const float* __restrict__ r, int d) {
  float s = -0.0f;
  if ((d & 3) == 0 && ((uintptr_t)r & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(r);
    for (int q = 0; q < d / 4; q++) {
      float4 v = __ldg(r4 + q);
      s = __fadd_rn(s, __fmul_rn(v.x, v.x));
      s = __fadd_rn(s, __fmul_rn(v.y, v.y));
      s = __fadd_rn(s, __fmul_rn(v.z, v.z));
      s = __fadd_rn(s, __fmul_rn(v.w, v.w));
    }
  } else {
    for (int t = 0; t < d; t++) {
      float v = __ldg(r + t);
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
  }
  return s;
}

__global__ void k_row_sumsq(const float* __restrict__ m, long rows, int d, float* __restrict__ out) {
  pdl_wait();
  long r = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) out[r] = row_sumsq(m + r * d, d);
}

// The same sums for d % 32 == 0, one thread per row with the row streamed
// through shared memory: R rows per one-warp block (32, or 8 when there are
// few rows, so that more warps keep loads in flight), 32-column slices copied
// with cp.async (8 slices in flight), 16-byte chunk q of row t at q ^ (t & 7)
// so that each thread's LDS.128 reads are free of bank conflicts.
constexpr int NS_ROWS = 32, NS_STAGES = 8;

template <int R>
__global__ void __launch_bounds__(32) k_row_sumsq_staged(const float* __restrict__ m, long rows,
                                                         int d, float* __restrict__ out) {
  pdl_wait();
  __shared__ __align__(16) float buf[NS_STAGES][R][32];
  const int t = threadIdx.x;
  const long r0 = (long)blockIdx.x * R;
  const int nsl = d / 32;
  auto issue = [&](int sl) {
    if (sl < nsl) {
#pragma unroll
      for (int u = 0; u < R / 4; u++) {
        const int r = u * 4 + (t >> 3), q = t & 7;
        const long row = min(r0 + r, rows - 1);
        const float* src = m + row * d + sl * 32 + q * 4;
        float* dst = &buf[sl % NS_STAGES][r][(q ^ (r & 7)) * 4];
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(dst)),
                     "l"(src)
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int s = 0; s < NS_STAGES - 1; s++) issue(s);
  float s = -0.0f;
  const int tr = t < R ? t : 0;  // lanes past R rows idle
  for (int sl = 0; sl < nsl; sl++) {
    issue(sl + NS_STAGES - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(NS_STAGES - 1) : "memory");
    __syncwarp();
    const float4* r4 = reinterpret_cast<const float4*>(buf[sl % NS_STAGES][tr]);
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const float4 v = r4[q ^ (tr & 7)];
      s = __fadd_rn(s, __fmul_rn(v.x, v.x));
      s = __fadd_rn(s, __fmul_rn(v.y, v.y));
      s = __fadd_rn(s, __fmul_rn(v.z, v.z));
      s = __fadd_rn(s, __fmul_rn(v.w, v.w));
    }
    __syncwarp();  // the slot is refilled next iteration
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (t < R && r0 + t < rows) out[r0 + t] = s;
}

__global__ void k_sel_sumsq(const float* __restrict__ x, long n, int d,
                            const uint32_t* __restrict__ ids, long r0, long r1,
                            float* __restrict__ out, uint32_t* status) {
  pdl_wait();
  long p = r0 + (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= r1) return;
  long row = ids ? (long)ids[p] : p;
  if (row >= n) {
    atomicOr(status, ST_BAD_ROW);
    out[p - r0] = 0.0f;
    return;
  }
  out[p - r0] = row_sumsq(x + row * d, d);
}

// faiss normalize_into for one row per thread (core/cpu.rs:219-230):
// divide by max |v| (zero rows keep 1), then by sqrt of the sequential sum of
// squares of the scaled row.
__global__ void k_normalize(const float* __restrict__ src, long rows, int d, float* __restrict__ dst) {
  pdl_wait();
  long r = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float* a = src + r * d;
  float mx = 0.0f;
  for (int t = 0; t < d; t++) mx = fmaxf(mx, fabsf(a[t]));
  float s = mx > 0.0f ? mx : 1.0f;
  float ss = -0.0f;
  for (int t = 0; t < d; t++) {
    float u = __fdiv_rn(a[t], s);
    ss = __fadd_rn(ss, __fmul_rn(u, u));
  }
  float nrm = __fsqrt_rn(ss);
  float s2 = nrm > 0.0f ? nrm : 1.0f;
  float* o = dst + r * d;
  for (int t = 0; t < d; t++) o[t] = __fdiv_rn(__fdiv_rn(a[t], s), s2);
}

// The EMA step, one block per centroid (core/cpu.rs:389-432).
__global__ void k_ema(float* __restrict__ pos, float* __restrict__ usage,
                      const float* __restrict__ sums, const uint32_t* __restrict__ counts, int d,
                      float a32, float decay, int replace) {
  pdl_wait();
  long j = blockIdx.x;
  float u = usage[j];
  uint32_t cnt = counts[j];
  float ud = replace ? u : __fmul_rn(u, decay);
  float mass = ud;
  if (cnt != 0) {
    float count = __uint2float_rn(cnt);
    float retained = replace ? 0.0f : ud;
    float step = __fmul_rn(a32, count);
    mass = __fadd_rn(retained, step);
    float w = __fdiv_rn(step, mass);
    float* c = pos + j * d;
    const float* s = sums + j * d;
    // Four elements per thread per round, their loads issued together.
    for (int t0 = threadIdx.x; t0 < d; t0 += 4 * blockDim.x) {
      float sv[4], cv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + u * blockDim.x;
        sv[u] = t < d ? s[t] : 0.0f;
        cv[u] = t < d ? c[t] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + u * blockDim.x;
        if (t < d) {
          const float mean = __fdiv_rn(sv[u], count);
          c[t] = w == 1.0f ? mean : __fadd_rn(cv[u], __fmul_rn(w, __fsub_rn(mean, cv[u])));
        }
      }
    }
  }
  __syncthreads();  // every thread has read usage[j]
  if (threadIdx.x == 0) usage[j] = mass;
}

// k_ema with 16-byte loads and stores (d % 4 == 0, aligned rows): one block
// per centroid, each thread four consecutive columns a round, the same
// per-element arithmetic.
__global__ void k_ema4(float* __restrict__ pos, float* __restrict__ usage,
                       const float* __restrict__ sums, const uint32_t* __restrict__ counts, int d,
                       float a32, float decay, int replace) {
  pdl_wait();
  const long j = blockIdx.x;
  const float u = usage[j];
  const uint32_t cnt = counts[j];
  const float ud = replace ? u : __fmul_rn(u, decay);
  float mass = ud;
  if (cnt != 0) {
    const float count = __uint2float_rn(cnt);
    const float retained = replace ? 0.0f : ud;
    const float step = __fmul_rn(a32, count);
    mass = __fadd_rn(retained, step);
    const float w = __fdiv_rn(step, mass);
    float4* c = reinterpret_cast<float4*>(pos + j * d);
    const float4* s = reinterpret_cast<const float4*>(sums + j * d);
    for (int q = threadIdx.x; q < d / 4; q += blockDim.x) {
      const float4 sv = s[q];
      float4 cv = c[q];
      auto one = [&](float sx, float cx) {
        const float mean = __fdiv_rn(sx, count);
        return w == 1.0f ? mean : __fadd_rn(cx, __fmul_rn(w, __fsub_rn(mean, cx)));
      };
      cv.x = one(sv.x, cv.x);
      cv.y = one(sv.y, cv.y);
      cv.z = one(sv.z, cv.z);
      cv.w = one(sv.w, cv.w);
      c[q] = cv;
    }
  }
  __syncthreads();  // every thread has read usage[j]
  if (threadIdx.x == 0) usage[j] = mass;
}

// The EMA step (k_ema's arithmetic, bit for bit) fused with the next step's
// readout of the updated centroid and the screen's summary of the centroids
// it will read (k_cent_max's words: max |c|, a bound on the row norm, a
// non-finite flag, under generation gen): the block holds the row in shared
// memory after the update. L2 (SPH false): readout[j] = the row's squared
// norm, sequential in column order (row_norms); the summary is of the row.
// Spherical: readout row j = faiss normalize_into of the row (k_normalize's
// arithmetic); the summary is of that normalised row. One block of 128
// threads per centroid; d + 32 floats of dynamic shared memory.
__device__ __forceinline__ unsigned long long summary_tag(uint32_t gen) {
  return (unsigned long long)gen << 32;
}
template <bool SPH>
__global__ void __launch_bounds__(128) k_ema_readout(
    float* __restrict__ pos, float* __restrict__ usage, const float* __restrict__ sums,
    const uint32_t* __restrict__ counts, int d, float a32, float decay, int replace,
    float* __restrict__ readout, unsigned long long* __restrict__ cinfo, uint32_t gen) {
  pdl_wait();
  extern __shared__ float row_s[];  // [d], then 32 floats of reduction slots
  float* red = row_s + d;
  const long j = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float u = usage[j];
  const uint32_t cnt = counts[j];
  const float ud = replace ? u : __fmul_rn(u, decay);
  float mass = ud;
  float* c = pos + j * d;
  if (cnt != 0) {
    const float count = __uint2float_rn(cnt);
    const float retained = replace ? 0.0f : ud;
    const float step = __fmul_rn(a32, count);
    mass = __fadd_rn(retained, step);
    const float w = __fdiv_rn(step, mass);
    const float* s = sums + j * d;
    for (int t = tid; t < d; t += blockDim.x) {
      const float mean = __fdiv_rn(s[t], count);
      const float cv = c[t];
      const float nv = w == 1.0f ? mean : __fadd_rn(cv, __fmul_rn(w, __fsub_rn(mean, cv)));
      c[t] = nv;
      row_s[t] = nv;
    }
  } else {
    for (int t = tid; t < d; t += blockDim.x) row_s[t] = c[t];
  }
  __syncthreads();  // the row is in shared memory; every thread has read usage[j]
  if (tid == 0) usage[j] = mass;
  // Max |v| and finiteness of the row, over the block.
  float mx = 0.0f;
  int fin = 1;
  for (int t = tid; t < d; t += blockDim.x) {
    const float v = row_s[t];
    fin &= isfinite(v) ? 1 : 0;
    mx = fmaxf(mx, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  fin = __all_sync(0xFFFFFFFFu, fin);
  if (lane == 0) {
    red[warp] = mx;
    red[8 + warp] = fin ? 1.0f : 0.0f;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w2 = 1; w2 < (int)(blockDim.x >> 5); w2++) {
      mx = fmaxf(mx, red[w2]);
      fin = fin && red[8 + w2] != 0.0f;
    }
    red[16] = mx;
    red[17] = fin ? 1.0f : 0.0f;
  }
  __syncthreads();
  mx = red[16];
  fin = red[17] != 0.0f;
  if (!SPH) {
    if (tid == 0) {
      float ss = -0.0f;
      for (int t = 0; t < d; t++) ss = __fadd_rn(ss, __fmul_rn(row_s[t], row_s[t]));
      readout[j] = ss;
      const unsigned long long tag = summary_tag(gen);
      if (!fin) {
        summary_max(&cinfo[2], tag | 1ull);
      } else {
        summary_max(&cinfo[0], tag | __float_as_uint(mx));
        summary_max(&cinfo[1], tag | __float_as_uint(sqrtf(ss) * (1.0f + 1.0f / 512.0f)));
      }
    }
  } else {
    const float sc = mx > 0.0f ? mx : 1.0f;
    if (tid == 0) {
      float ss = -0.0f;
      for (int t = 0; t < d; t++) {
        const float q = __fdiv_rn(row_s[t], sc);
        ss = __fadd_rn(ss, __fmul_rn(q, q));
      }
      const float nrm = __fsqrt_rn(ss);
      red[18] = nrm > 0.0f ? nrm : 1.0f;
    }
    __syncthreads();
    const float s2 = red[18];
    float* o = readout + j * d;
    float omx = 0.0f, oss = 0.0f;
    int ofin = 1;
    for (int t = tid; t < d; t += blockDim.x) {
      const float v = __fdiv_rn(__fdiv_rn(row_s[t], sc), s2);
      o[t] = v;
      ofin &= isfinite(v) ? 1 : 0;
      omx = fmaxf(omx, fabsf(v));
      oss = fmaf(v, v, oss);
    }
#pragma unroll
    for (int q = 16; q >= 1; q >>= 1) {
      omx = fmaxf(omx, __shfl_xor_sync(0xFFFFFFFFu, omx, q));
      oss += __shfl_xor_sync(0xFFFFFFFFu, oss, q);
    }
    ofin = __all_sync(0xFFFFFFFFu, ofin);
    __syncthreads();  // red[16..18] are no longer read
    if (lane == 0) {
      red[warp] = omx;
      red[8 + warp] = oss;
      red[16 + warp] = ofin ? 1.0f : 0.0f;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w2 = 1; w2 < (int)(blockDim.x >> 5); w2++) {
        omx = fmaxf(omx, red[w2]);
        oss += red[8 + w2];
        ofin = ofin && red[16 + w2] != 0.0f;
      }
      const unsigned long long tag = summary_tag(gen);
      if (!ofin) {
        summary_max(&cinfo[2], tag | 1ull);
      } else {
        summary_max(&cinfo[0], tag | __float_as_uint(omx));
        summary_max(&cinfo[1], tag | __float_as_uint(sqrtf(oss) * (1.0f + 1.0f / 512.0f)));
      }
    }
  }
}

// Revival splits, one block per (donor, dead) pair (core/mod.rs:374-399).
__global__ void k_split(float* __restrict__ pos, float* __restrict__ usage,
                        const uint32_t* __restrict__ pairs, int d) {
  pdl_wait();
  uint32_t s = pairs[2 * blockIdx.x], t = pairs[2 * blockIdx.x + 1];
  const float eps = (float)1e-4;
  float* cs = pos + (long)s * d;
  float* ct = pos + (long)t * d;
  bool same = true;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float off = __fmul_rn(eps, (i % 2 == 0) ? 1.0f : -1.0f);
    float c = cs[i];
    float dn = __fmul_rn(c, __fsub_rn(1.0f, off));
    float ch = __fmul_rn(c, __fadd_rn(1.0f, off));
    same = same && (dn == ch);
  }
  int all_same = __syncthreads_and(same ? 1 : 0);
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float off = __fmul_rn(eps, (i % 2 == 0) ? 1.0f : -1.0f);
    float c = cs[i];
    float dn = __fmul_rn(c, __fsub_rn(1.0f, off));
    float ch = __fmul_rn(c, __fadd_rn(1.0f, off));
    if (i == 0 && all_same) {
      float up = nextafterf(ch, INFINITY);
      ch = isfinite(up) ? up : nextafterf(ch, -INFINITY);
    }
    cs[i] = dn;
    ct[i] = ch;
  }
  if (threadIdx.x == 0) {
    float half = __fdiv_rn(usage[s], 2.0f);
    usage[s] = half;
    usage[t] = half;
  }
}

// ---- deterministic scatter-add: a stable counting sort by label, then one
// sequential f32 sum per (centroid, column) in selection order.

// The positions are cut into segments; a segment's positions are ranked
// among the segment's positions with the same label (stable), the segment's
// per-label counts are scanned over the segments per label, the labels'
// totals are scanned over the labels, and each position lands at
// start[label] + (its label's count in earlier segments) + its rank.
// Two segment shapes: with k <= kRankSmem a block of eight warps ranks
// kBlockSeg positions in shared-memory histograms (one per warp, combined
// in warp order), so the per-(segment, label) table has one row per 2,048
// positions; with larger k one warp ranks kSeg positions with its counts in
// global memory (the caller zeroes them).
constexpr int kSeg = 256;  // positions a warp ranks
constexpr int kRankWarps = 8;
constexpr int kBlockSeg = kSeg * kRankWarps;  // positions a block ranks (k <= kRankSmem)
constexpr uint32_t kRankSmem = 1024;

// In-warp stable ranks of the warp's kSeg positions starting at p0, counted
// in cnt (shared or global; only the warp touches it). lab[] receives the
// labels (0xFFFFFFFF past the end or for a bad label), rk[] the ranks.
__device__ __forceinline__ void warp_rank(const uint32_t* __restrict__ labels, long r0, long m,
                                          long p0, uint32_t k, uint32_t* cnt,
                                          uint32_t (&lab)[kSeg / 32], uint32_t (&rk)[kSeg / 32],
                                          uint32_t* status) {
  const int lane = threadIdx.x & 31;
  // The segment's labels for this lane, all loads in flight together.
#pragma unroll
  for (int c = 0; c < kSeg / 32; c++) {
    const long p = p0 + c * 32 + lane;
    lab[c] = p < m ? labels[r0 + p] : 0xFFFFFFFFu;
  }
#pragma unroll
  for (int c = 0; c < kSeg / 32; c++) {
    const long p = p0 + c * 32 + lane;
    const uint32_t l = lab[c];
    const bool valid = l < k;
    if (p < m && !valid) atomicOr(status, ST_BAD_LABEL);
    if (!valid) lab[c] = 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xFFFFFFFFu, valid ? l : 0xFFFFFFFFu);
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (valid && lane == leader) {
      base = cnt[l];
      cnt[l] = base + __popc(peers);
    }
    base = __shfl_sync(0xFFFFFFFFu, base, leader);
    rk[c] = base + __popc(peers & ((1u << lane) - 1u));
    __syncwarp();
  }
}

// k > kRankSmem: one warp per kSeg positions, counts in segcnt (zeroed by
// the caller; only the segment's warp updates its row).
__global__ void __launch_bounds__(256) k_seg_rank(const uint32_t* __restrict__ labels, long r0,
                                                  long m, uint32_t k,
                                                  uint32_t* __restrict__ segcnt,
                                                  uint32_t* __restrict__ rank, uint32_t* status) {
  pdl_wait();
  const long seg = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const long segs = (m + kSeg - 1) / kSeg;
  if (seg >= segs) return;
  uint32_t lab[kSeg / 32], rk[kSeg / 32];
  warp_rank(labels, r0, m, seg * kSeg, k, segcnt + seg * (long)k, lab, rk, status);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < kSeg / 32; c++)
    if (lab[c] != 0xFFFFFFFFu) rank[seg * kSeg + c * 32 + lane] = rk[c];
}

// k <= kRankSmem: one block of kRankWarps warps per kBlockSeg positions.
// Each warp ranks its kSeg positions in its own shared histogram; the
// histograms are then turned into each warp's offset per label (exclusive,
// in warp order, so the ranks stay stable) and the block's totals go out as
// the segment's row of segcnt (every entry written: no zeroing pass).
__global__ void __launch_bounds__(kRankWarps * 32) k_block_rank(
    const uint32_t* __restrict__ labels, long r0, long m, uint32_t k,
    uint32_t* __restrict__ segcnt, uint32_t* __restrict__ rank, uint32_t* status) {
  pdl_wait();
  __shared__ uint32_t hist[kRankWarps][kRankSmem];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long seg = blockIdx.x;
  for (uint32_t l = lane; l < k; l += 32) hist[w][l] = 0;
  __syncwarp();
  uint32_t lab[kSeg / 32], rk[kSeg / 32];
  const long p0 = seg * kBlockSeg + (long)w * kSeg;
  warp_rank(labels, r0, m, p0, k, hist[w], lab, rk, status);
  __syncthreads();
  for (uint32_t l = threadIdx.x; l < k; l += blockDim.x) {
    uint32_t off = 0;
#pragma unroll
    for (int v = 0; v < kRankWarps; v++) {
      const uint32_t t = hist[v][l];
      hist[v][l] = off;
      off += t;
    }
    segcnt[seg * (long)k + l] = off;
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kSeg / 32; c++)
    if (lab[c] != 0xFFFFFFFFu) rank[p0 + c * 32 + lane] = rk[c] + hist[w][lab[c]];
}

// Exclusive scan of counts into start[0..k] by one block of kScanThreads
// threads, and the labels grouped by the size of their count, largest first
// (bucket b = bit length of the count), into by_size[0..k), so that the
// segment sums start the longest chains in the first wave (a chain is
// sequential, and the largest one sets the kernel's length). Only the launch
// order of the sum blocks depends on by_size: the order within a bucket is
// the order of the shared-memory atomics, and every sum comes out the same.
// counts were written by other blocks of the grid: read through L2.
constexpr int kScanThreads = 256;
__device__ void label_scan_block(const uint32_t* counts, uint32_t k, uint32_t* __restrict__ start,
                                 uint32_t* __restrict__ by_size) {
  __shared__ uint32_t part[kScanThreads];
  __shared__ uint32_t bins[34];
  if (threadIdx.x < 34) bins[threadIdx.x] = 0;
  const uint32_t per = (k + kScanThreads - 1) / kScanThreads;
  const uint32_t lo = min(threadIdx.x * per, k), hi = min(lo + per, k);
  uint32_t s = 0;
  for (uint32_t l = lo; l < hi; l++) s += __ldcg(counts + l);
  part[threadIdx.x] = s;
  __syncthreads();
  for (uint32_t l = lo; l < hi; l++) atomicAdd(&bins[32 - __clz(__ldcg(counts + l))], 1u);
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const uint32_t v = threadIdx.x >= (unsigned)off ? part[threadIdx.x - off] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  uint32_t run = threadIdx.x ? part[threadIdx.x - 1] : 0;
  for (uint32_t l = lo; l < hi; l++) {
    start[l] = run;
    run += __ldcg(counts + l);
  }
  if (threadIdx.x == kScanThreads - 1) start[k] = part[threadIdx.x];
  if (threadIdx.x == 0) {
    // Bucket starts, largest bucket (32: counts of 2^31 or more) first.
    uint32_t acc = 0;
    for (int bb = 32; bb >= 0; bb--) {
      const uint32_t c = bins[bb];
      bins[bb] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (uint32_t l = lo; l < hi; l++)
    by_size[atomicAdd(&bins[32 - __clz(__ldcg(counts + l))], 1u)] = l;
}

// Per label: exclusive prefix of its counts over segments (in place), and
// the label's total. One warp per label: in each round lane l reads a run of
// kScanR consecutive segments (all loads in flight together), the warp scans
// the runs' sums, and each lane writes its run's prefixes. The block that
// finishes last (a ticket taken after each block's counts are fenced; no
// block waits for another) then runs the label scan, and resets the ticket
// for the next call.
constexpr int kScanR = 16;
__global__ void __launch_bounds__(kScanThreads) k_seg_scan(
    uint32_t* __restrict__ segcnt, long segs, uint32_t k, uint32_t* counts,
    uint32_t* __restrict__ start, uint32_t* __restrict__ by_size, uint32_t* ticket) {
  pdl_wait();
  const uint32_t l = (uint32_t)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (l < k) {  // the whole warp: its lanes share l
    uint32_t carry = 0;
    for (long s0 = 0; s0 < segs; s0 += 32 * kScanR) {
      const long my0 = s0 + (long)lane * kScanR;
      uint32_t c[kScanR];
      uint32_t sum = 0;
#pragma unroll
      for (int r = 0; r < kScanR; r++) {
        c[r] = my0 + r < segs ? segcnt[(my0 + r) * k + l] : 0u;
        sum += c[r];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t run = carry + incl - sum;
#pragma unroll
      for (int r = 0; r < kScanR; r++) {
        if (my0 + r < segs) segcnt[(my0 + r) * k + l] = run;
        run += c[r];
      }
      carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) {
      counts[l] = carry;
      __threadfence();
    }
  }
  __shared__ uint32_t last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  label_scan_block(counts, k, start, by_size);
  if (threadIdx.x == 0) *ticket = 0;
}

// Place every position at its sorted slot; the slot holds the data row id.
// seg_len: positions per segment of segcnt's rows (kSeg or kBlockSeg).
__global__ void k_place(const uint32_t* __restrict__ labels, const uint32_t* __restrict__ ids,
                        long r0, long m, long n, uint32_t k, int seg_len,
                        const uint32_t* __restrict__ segcnt, const uint32_t* __restrict__ start,
                        const uint32_t* __restrict__ rank, uint32_t* __restrict__ order,
                        uint32_t* status) {
  pdl_wait();
  long p = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= m) return;
  uint32_t l = labels[r0 + p];
  if (l >= k) return;
  long seg = p / seg_len;
  uint32_t row = ids ? ids[r0 + p] : (uint32_t)(r0 + p);
  if ((long)row >= n) {
    atomicOr(status, ST_BAD_ROW);
    row = 0;
  }
  order[start[l] + segcnt[seg * k + l] + rank[p]] = row;
}

// s += x[ord[i] * d] for i = 0 .. n-1 in order: batches of Q rows, the next
// batch's loads issued before the current batch is added, then one row at a
// time.
template <int Q>
__device__ __forceinline__ float chain_sum(const float* __restrict__ xt, const uint32_t* ord,
                                           uint32_t n, int d, float s) {
  uint32_t i = 0;
  float v[Q];
  if (n >= (uint32_t)Q) {
#pragma unroll
    for (int q = 0; q < Q; q++) v[q] = __ldg(xt + (long)ord[q] * d);
  }
  for (; i + 2 * Q <= n; i += Q) {
    float w[Q];
#pragma unroll
    for (int q = 0; q < Q; q++) w[q] = __ldg(xt + (long)ord[i + Q + q] * d);
#pragma unroll
    for (int q = 0; q < Q; q++) s = __fadd_rn(s, v[q]);
#pragma unroll
    for (int q = 0; q < Q; q++) v[q] = w[q];
  }
  if (i + Q <= n) {
#pragma unroll
    for (int q = 0; q < Q; q++) s = __fadd_rn(s, v[q]);
    i += Q;
  }
  for (; i < n; i++) s = __fadd_rn(s, __ldg(xt + (long)ord[i] * d));
  return s;
}

// sums[j][t] = rows of centroid j added in selection order from +0;
// acc[j][t] += sums[j][t]. One thread per (centroid, column); block b takes
// the b / cb-th largest centroid (by_size) and its column block b % cb, so
// that the longest chains are scheduled first. The block stages
// its centroid's row ids in shared memory, kSumStage at a time, and each
// thread keeps the next 32 rows' loads in flight while it adds the current 32
// in order (the adds of one column form one sequential chain, and the
// largest centroid's chain sets the kernel's length: measured on C2's full
// pass, 0.24 ms with 16-row batches, 0.20 ms with 32, 0.21 ms with 64).
constexpr uint32_t kSumStage = 1024;
__global__ void __launch_bounds__(128) k_seg_sum(const float* __restrict__ x, int d, int cb,
                                                 const uint32_t* __restrict__ order,
                                                 const uint32_t* __restrict__ start,
                                                 const uint32_t* __restrict__ by_size,
                                                 float* __restrict__ sums,
                                                 float* __restrict__ acc) {
  pdl_wait();
  __shared__ uint32_t ord_s[kSumStage];
  const long j = by_size[blockIdx.x / cb];
  const int t = (blockIdx.x % cb) * blockDim.x + threadIdx.x;
  const bool active = t < d;
  const float* xt = x + (active ? t : 0);
  const uint32_t b = start[j], e = start[j + 1];
  float s = 0.0f;
  for (uint32_t c0 = b; c0 < e; c0 += kSumStage) {
    const uint32_t n = min(e - c0, kSumStage);
    __syncthreads();  // the last chunk's ids are no longer read
    for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) ord_s[u] = order[c0 + u];
    __syncthreads();
    if (!active) continue;
    s = chain_sum<32>(xt, ord_s, n, d, s);
  }
  if (active) {
    sums[j * d + t] = s;
    if (acc) acc[j * d + t] = __fadd_rn(acc[j * d + t], s);
  }
}

// The same with the rows streamed through shared memory (d % 4 == 0, 16-byte
// aligned rows): a block takes one centroid and a 128-column slice, copies
// R rows' slices at a time with cp.async (NS stages in flight, each thread
// moving 16-byte chunks; the centroid's row ids staged ID at a time), and
// each thread adds its column of every staged row in selection order: the
// scalar kernel's chain bit for bit. The loads no longer wait on the chain,
// so the longest centroid's chain (which sets the kernel's length) runs at
// shared-memory speed. Two shapes: 32 rows x 4 stages (64 KB, three blocks
// an SM) when the centroids average many rows (a full pass), 16 rows x 2
// stages (16 KB, thirteen blocks an SM) for a training batch, whose
// centroids average a few rows and whose blocks are mostly start-up.
constexpr int SS_C = 128;
template <int R, int NS>
constexpr size_t ss_smem() {
  return (size_t)NS * R * SS_C * sizeof(float);
}
template <int R, int NS, int ID>
__global__ void __launch_bounds__(SS_C) k_seg_sum_staged(
    const float* __restrict__ x, int d, int cb, const uint32_t* __restrict__ order,
    const uint32_t* __restrict__ start, const uint32_t* __restrict__ by_size,
    float* __restrict__ sums, float* __restrict__ acc) {
  pdl_wait();
  extern __shared__ __align__(16) float ss_buf[];  // [NS][R][SS_C]
  __shared__ uint32_t ord_s[ID];
  const long j = by_size[blockIdx.x / cb];
  const int col0 = (blockIdx.x % cb) * SS_C;
  const int t = threadIdx.x;
  const bool active = col0 + t < d;
  const uint32_t b = start[j], e = start[j + 1];
  float s = 0.0f;
  for (uint32_t c0 = b; c0 < e; c0 += ID) {
    const uint32_t n = min(e - c0, (uint32_t)ID);
    __syncthreads();  // the last chunk's ids and rows are no longer read
    for (uint32_t u = t; u < n; u += SS_C) ord_s[u] = order[c0 + u];
    __syncthreads();
    const int nst = (int)((n + R - 1) / R);
    auto issue = [&](int st) {
      if (st < nst) {
        float* buf = ss_buf + (st % NS) * R * SS_C;
        const uint32_t r0 = (uint32_t)st * R;
#pragma unroll
        for (int u = 0; u < R / 4; u++) {  // R / 4 chunks a thread
          const int idx = u * SS_C + t;
          const int r = idx / (SS_C / 4), q = idx % (SS_C / 4);
          const int col = col0 + q * 4;
          if (r0 + r < n && col < d) {
            const float* src = x + (long)ord_s[r0 + r] * d + col;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                             (uint32_t)__cvta_generic_to_shared(buf + r * SS_C + q * 4)),
                         "l"(src)
                         : "memory");
          }
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int st = 0; st < NS - 1; st++) issue(st);
    for (int st = 0; st < nst; st++) {
      issue(st + NS - 1);
      asm volatile("cp.async.wait_group %0;" ::"n"(NS - 1) : "memory");
      __syncthreads();
      const float* buf = ss_buf + (st % NS) * R * SS_C + t;
      const int rows = min(R, (int)(n - (uint32_t)st * R));
      if (active) {
        if (rows == R) {
#pragma unroll
          for (int r = 0; r < R; r++) s = __fadd_rn(s, buf[r * SS_C]);
        } else {
          for (int r = 0; r < rows; r++) s = __fadd_rn(s, buf[r * SS_C]);
        }
      }
      __syncthreads();  // the stage is refilled next iteration
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  if (active) {
    sums[j * d + col0 + t] = s;
    if (acc) acc[j * d + col0 + t] = __fadd_rn(acc[j * d + col0 + t], s);
  }
}

// Count of every label among labels[0 .. m) into cnt (zeroed by the caller);
// per-block shared-memory histograms when k is small. Integer counts: the
// order of the additions does not matter.
constexpr uint32_t kHistSmem = 4096;
__global__ void k_label_hist(const uint32_t* __restrict__ labels, long m, uint32_t k,
                             uint32_t* __restrict__ cnt) {
  pdl_wait();
  __shared__ uint32_t h[kHistSmem];
  const bool sm = k <= kHistSmem;
  if (sm) {
    for (uint32_t l = threadIdx.x; l < k; l += blockDim.x) h[l] = 0;
    __syncthreads();
  }
  for (long p = (long)blockIdx.x * blockDim.x + threadIdx.x; p < m;
       p += (long)gridDim.x * blockDim.x) {
    const uint32_t l = labels[p];
    if (l < k) atomicAdd(sm ? &h[l] : &cnt[l], 1u);
  }
  if (sm) {
    __syncthreads();
    for (uint32_t l = threadIdx.x; l < k; l += blockDim.x)
      if (h[l]) atomicAdd(&cnt[l], h[l]);
  }
}

// closing_means before the spherical renormalisation (core/mod.rs:404-429):
// a centroid with rows in the closing pass takes sums / (float)count, one
// without keeps its position.
__global__ void k_closing(const float* __restrict__ pos, const float* __restrict__ sums,
                          const uint32_t* __restrict__ cnt, long k, int d,
                          float* __restrict__ out) {
  pdl_wait();
  const long j = blockIdx.x;
  const uint32_t c = cnt[j];
  const float nf = __uint2float_rn(c);
  for (int t = threadIdx.x; t < d; t += blockDim.x) {
    const long q = j * d + t;
    out[q] = c > 0 ? __fdiv_rn(sums[q], nf) : pos[q];
  }
}

unsigned blocks_for(size_t n, unsigned per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

void row_norms(eb_engine* e, const float* m, size_t rows, size_t d, float* out) {
  if (rows == 0) return;
  if (d % 32 == 0 && ((uintptr_t)m & 15) == 0) {
    if (rows <= (size_t)e->num_sms * 32)
      launch_pdl(e, k_row_sumsq_staged<8>, blocks_for(rows, 8), 32, 0, m, (long)rows, (int)d, out);
    else
      launch_pdl(e, k_row_sumsq_staged<NS_ROWS>, blocks_for(rows, NS_ROWS), 32, 0, m, (long)rows,
                                                                                  (int)d, out);
  } else {
    launch_pdl(e, k_row_sumsq, blocks_for(rows, kRowThreads), kRowThreads, 0, m, (long)rows,
                                                                              (int)d, out);
  }
  EB_LAUNCH("row_norms");
}

void sel_row_norms(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* ids,
                   size_t r0, size_t r1, float* out) {
  if (r1 <= r0) return;
  launch_pdl(e, k_sel_sumsq, blocks_for(r1 - r0, kRowThreads), kRowThreads, 0, x, (long)n, (int)d, ids, (long)r0, (long)r1, out, e->d_status);
  EB_LAUNCH("sel_row_norms");
}

void normalize_rows(eb_engine* e, const float* src, size_t rows, size_t d, float* dst) {
  if (rows == 0) return;
  launch_pdl(e, k_normalize, blocks_for(rows, kRowThreads), kRowThreads, 0, src, (long)rows,
                                                                            (int)d, dst);
  EB_LAUNCH("normalize_rows");
}

void label_counts(eb_engine* e, const uint32_t* labels, size_t m, size_t k, uint32_t* cnt) {
  EB_CUDA(cudaMemsetAsync(cnt, 0, k * sizeof(uint32_t), e->stream));
  if (m == 0) return;
  const unsigned grid = (unsigned)std::min<size_t>(blocks_for(m, 256), (size_t)e->num_sms * 2);
  launch_pdl(e, k_label_hist, grid, 256, 0, labels, (long)m, (uint32_t)k, cnt);
  EB_LAUNCH("label_counts");
}

void closing_means(eb_engine* e, const float* pos, const float* sums, const uint32_t* cnt,
                   size_t k, size_t d, float* out) {
  if (k == 0) return;
  launch_pdl(e, k_closing, (unsigned)k, 128, 0, pos, sums, cnt, (long)k, (int)d, out);
  EB_LAUNCH("closing_means");
}

void ema_update(eb_engine* e, float* pos, float* usage, const float* sums, const uint32_t* counts,
                size_t k, size_t d, float alpha, float decay, bool replace) {
  if (k == 0) return;
  if (d % 4 == 0 && ((uintptr_t)pos & 15) == 0 && ((uintptr_t)sums & 15) == 0) {
    const unsigned q = (unsigned)(d / 4);
    const unsigned threads = q >= 256 ? 256 : (q + 31) / 32 * 32;
    launch_pdl(e, k_ema4, (unsigned)k, threads, 0, pos, usage, sums, counts, (int)d, alpha,
               decay, replace ? 1 : 0);
  } else {
    launch_pdl(e, k_ema, (unsigned)k, 128, 0, pos, usage, sums, counts, (int)d, alpha, decay,
               replace ? 1 : 0);
  }
  EB_LAUNCH("ema_update");
}

bool ema_update_readout(eb_engine* e, float* pos, float* usage, const float* sums,
                        const uint32_t* counts, size_t k, size_t d, float alpha, float decay,
                        bool replace, bool spherical, float* readout,
                        unsigned long long* cinfo, uint32_t gen) {
  const size_t smem = (d + 32) * sizeof(float);
  if (k == 0 || smem > 48 * 1024) return false;
  if (spherical)
    launch_pdl(e, k_ema_readout<true>, (unsigned)k, 128, smem, pos, usage, sums, counts, (int)d,
               alpha, decay, replace ? 1 : 0, readout, cinfo, gen);
  else
    launch_pdl(e, k_ema_readout<false>, (unsigned)k, 128, smem, pos, usage, sums, counts, (int)d,
               alpha, decay, replace ? 1 : 0, readout, cinfo, gen);
  EB_LAUNCH("ema_update + readout");
  return true;
}

void split(eb_engine* e, float* pos, float* usage, const uint32_t* d_pairs, size_t npairs,
           size_t d) {
  if (npairs == 0) return;
  launch_pdl(e, k_split, (unsigned)npairs, 128, 0, pos, usage, d_pairs, (int)d);
  EB_LAUNCH("split");
}

void label_order(eb_engine* e, const uint32_t* ids, size_t r0, size_t r1, size_t n,
                 const uint32_t* labels, size_t k, uint32_t* counts, const uint32_t** order_out,
                 const uint32_t** start_out, const uint32_t** by_size_out) {
  size_t m = r1 - r0;
  const bool block_rank = m > 0 && k <= kRankSmem;
  const size_t seg_len = block_rank ? kBlockSeg : kSeg;
  size_t segs = (m + seg_len - 1) / seg_len;
  if (segs == 0) segs = 1;
  uint32_t* segcnt = e->scratch_get<uint32_t>("sc_segcnt", segs * k);
  uint32_t* rank = e->scratch_get<uint32_t>("sc_rank", m ? m : 1);
  uint32_t* start = e->scratch_get<uint32_t>("sc_start", k + 1);
  uint32_t* order = e->scratch_get<uint32_t>("sc_order", m ? m : 1);
  uint32_t* by_size = e->scratch_get<uint32_t>("sc_by_size", k);
  uint32_t* ticket = e->scratch_get<uint32_t>("sc_ticket", 1, true);
  if (!block_rank) EB_CUDA(cudaMemsetAsync(segcnt, 0, segs * k * sizeof(uint32_t), e->stream));
  if (block_rank) {
    launch_pdl(e, k_block_rank, (unsigned)segs, kRankWarps * 32, 0, labels, (long)r0, (long)m,
               (uint32_t)k, segcnt, rank, e->d_status);
    EB_LAUNCH("scatter rank");
  } else if (m > 0) {
    const int warps = 8;
    launch_pdl(e, k_seg_rank, blocks_for(segs, warps), warps * 32, 0, labels, (long)r0, (long)m,
               (uint32_t)k, segcnt, rank, e->d_status);
    EB_LAUNCH("scatter rank");
  }
  launch_pdl(e, k_seg_scan, blocks_for(k * 32, kScanThreads), kScanThreads, 0, segcnt,
             (long)segs, (uint32_t)k, counts, start, by_size, ticket);
  EB_LAUNCH("scatter seg scan");
  if (m > 0) {
    launch_pdl(e, k_place, blocks_for(m, 256), 256, 0, labels, ids, (long)r0, (long)m, (long)n,
               (uint32_t)k, (int)seg_len, segcnt, start, rank, order, e->d_status);
    EB_LAUNCH("scatter place");
  }
  *order_out = order;
  *start_out = start;
  if (by_size_out) *by_size_out = by_size;
}

template <int R, int NS, int ID>
static void launch_seg_sum_staged(eb_engine* e, unsigned grid, const float* x, size_t d,
                                  unsigned cb, const uint32_t* order, const uint32_t* start,
                                  const uint32_t* by_size, float* sums, float* acc) {
  static uint64_t done = 0;  // one instance per shape
  if (!(done >> e->device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_seg_sum_staged<R, NS, ID>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)ss_smem<R, NS>()));
    done |= 1ull << e->device;
  }
  launch_pdl(e, k_seg_sum_staged<R, NS, ID>, grid, SS_C, ss_smem<R, NS>(), x, (int)d, (int)cb,
             order, start, by_size, sums, acc);
}

void scatter_add(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0,
                 size_t r1, const uint32_t* labels, size_t k, float* sums, uint32_t* counts,
                 float* acc) {
  const uint32_t *order, *start, *by_size;
  label_order(e, ids, r0, r1, n, labels, k, counts, &order, &start, &by_size);
  const bool vec = d % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)sums & 15) == 0 &&
                   (!acc || ((uintptr_t)acc & 15) == 0);
  if (vec) {
    const unsigned cb = blocks_for(d, SS_C);
    if (r1 - r0 <= 48 * k)  // a few rows a centroid on average
      launch_seg_sum_staged<16, 2, 256>(e, (unsigned)(k * cb), x, d, cb, order, start, by_size,
                                        sums, acc);
    else
      launch_seg_sum_staged<32, 4, 1024>(e, (unsigned)(k * cb), x, d, cb, order, start, by_size,
                                         sums, acc);
  } else {
    const unsigned cb = blocks_for(d, 128);
    launch_pdl(e, k_seg_sum, (unsigned)(k * cb), 128, 0, x, (int)d, (int)cb, order, start,
               by_size, sums, acc);
  }
  EB_LAUNCH("scatter sum");
}

}  // namespace eb

// ---- multi-GPU batch exchange: (labels, scores) slices through one staging
// buffer of world x 2s words, all-gathered in place between pack and unpack.

namespace eb {
namespace {

__global__ void k_shard_pack(const uint32_t* __restrict__ labels, const float* __restrict__ scores,
                             long len, long s, uint32_t* __restrict__ stage) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= s) return;
  stage[i] = i < len ? labels[i] : 0u;
  stage[s + i] = i < len ? __float_as_uint(scores[i]) : 0u;
}

__global__ void k_shard_unpack(const uint32_t* __restrict__ stage, long total, long s,
                               long soff, long stride, uint32_t* __restrict__ labels,
                               float* __restrict__ scores) {
  pdl_wait();
  const long p = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= total) return;
  const long q = p / s, i = p - q * s;
  labels[p] = stage[q * stride + i];
  scores[p] = __uint_as_float(stage[q * stride + soff + i]);
}

// The ranks' partial sums added in rank order, one thread per (centroid,
// column) word of the k x d block (plus the k counts); 16-byte loads and
// stores where the shares allow.
template <bool V4>
__global__ void k_reduce_partials(const uint32_t* __restrict__ stage, long stride, int world,
                                  long cnt_off, long sum_off, long k, long kd,
                                  float* __restrict__ sums, uint32_t* __restrict__ counts,
                                  float* __restrict__ acc) {
  pdl_wait();
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (V4) {
    const long q = t * 4;
    if (q < kd) {
      float4 s = *reinterpret_cast<const float4*>(stage + sum_off + q);
      for (int r = 1; r < world; r++) {
        const float4 v = *reinterpret_cast<const float4*>(stage + r * stride + sum_off + q);
        s.x = __fadd_rn(s.x, v.x);
        s.y = __fadd_rn(s.y, v.y);
        s.z = __fadd_rn(s.z, v.z);
        s.w = __fadd_rn(s.w, v.w);
      }
      *reinterpret_cast<float4*>(sums + q) = s;
      if (acc) {
        float4 a = *reinterpret_cast<float4*>(acc + q);
        a.x = __fadd_rn(a.x, s.x);
        a.y = __fadd_rn(a.y, s.y);
        a.z = __fadd_rn(a.z, s.z);
        a.w = __fadd_rn(a.w, s.w);
        *reinterpret_cast<float4*>(acc + q) = a;
      }
    }
  } else {
    for (long q = t; q < kd; q += (long)gridDim.x * blockDim.x) {
      float s = __uint_as_float(stage[sum_off + q]);
      for (int r = 1; r < world; r++) s = __fadd_rn(s, __uint_as_float(stage[r * stride + sum_off + q]));
      sums[q] = s;
      if (acc) acc[q] = __fadd_rn(acc[q], s);
    }
  }
  if (t < k) {
    uint32_t c = 0;
    for (int r = 0; r < world; r++) c += stage[r * stride + cnt_off + t];
    counts[t] = c;
  }
}

}  // namespace

void shard_pack(eb_engine* e, const uint32_t* labels, const float* scores, size_t len,
                size_t soff, size_t stride, uint32_t* stage) {
  if (soff == 0) return;
  launch_pdl(e, k_shard_pack, blocks_for(soff, 256), 256, 0, labels, scores, (long)len,
             (long)soff, stage + (size_t)e->rank * stride);
  EB_LAUNCH("shard_pack");
}

void shard_unpack(eb_engine* e, const uint32_t* stage, size_t total, size_t s, size_t soff,
                  size_t stride, uint32_t* labels, float* scores) {
  if (total == 0) return;
  launch_pdl(e, k_shard_unpack, blocks_for(total, 256), 256, 0, stage, (long)total, (long)s,
             (long)soff, (long)stride, labels, scores);
  EB_LAUNCH("shard_unpack");
}

void reduce_partials(eb_engine* e, const uint32_t* stage, size_t stride, int world,
                     size_t cnt_off, size_t sum_off, size_t k, size_t d, float* sums,
                     uint32_t* counts, float* acc) {
  const size_t kd = k * d;
  if (kd == 0) return;
  const bool v4 = kd % 4 == 0 && stride % 4 == 0 && sum_off % 4 == 0 &&
                  ((uintptr_t)stage & 15) == 0 && ((uintptr_t)sums & 15) == 0 &&
                  (!acc || ((uintptr_t)acc & 15) == 0);
  const size_t threads = std::max(v4 ? kd / 4 : std::min<size_t>(kd, (size_t)e->num_sms * 1024), k);
  if (v4)
    launch_pdl(e, k_reduce_partials<true>, blocks_for(threads, 256), 256, 0, stage, (long)stride,
               world, (long)cnt_off, (long)sum_off, (long)k, (long)kd, sums, counts, acc);
  else
    launch_pdl(e, k_reduce_partials<false>, blocks_for(threads, 256), 256, 0, stage, (long)stride,
               world, (long)cnt_off, (long)sum_off, (long)k, (long)kd, sums, counts, acc);
  EB_LAUNCH("reduce_partials");
}

}  // namespace eb

// ---- the group's peer-memory all-gather (a compute step's results pushed
// straight into every rank's copy of a symmetric exchange region over
// NVLink; nccl.cpp sets the regions up).

namespace eb {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t px_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Flag v has reached epoch (32-bit wrap-around order).
__device__ __forceinline__ bool px_reached(uint32_t v, uint32_t epoch) {
  return (int32_t)(v - epoch) >= 0;
}
constexpr uint64_t kPxWaitNs = 2000000000ull;  // every wait gives up after 2 s

// Region of rank q (peers[q], mapped on this GPU): flag words, then data.
// ready[r] (word r) and done[r] (word 64 + r) are written by rank r with the
// call's epoch; word 128 counts this kernel's finished blocks, word 129 is
// set by a block whose wait ran out.
// 1. Block 0 posts ready to every peer; every block waits (bounded) until
//    every peer has posted it: all ranks have reached this call, so no rank
//    still reads a region's previous contents.
// 2. The blocks push this rank's share (data words rank * words .. + words)
//    into the same place of every peer's region (16-byte stores).
// 3. Each block fences its stores at system scope and takes a ticket; the
//    last block posts done to every peer and waits (bounded) until every
//    peer has posted done here: then every share is in this rank's region.
// A wait that runs out sets ST_WAIT_TIMEOUT (the next sync reports it). A
// block whose entry wait ran out pushes nothing but still takes its ticket
// (so the count is whole for the next call), and then the last block posts
// no done: the peers' exit waits run out and report it too, rather than
// reading shares that were never sent.
__global__ void __launch_bounds__(256) k_px_allgather(uint32_t* const* __restrict__ peers,
                                                      int world, int rank, long words,
                                                      uint32_t epoch, uint32_t* status) {
  pdl_wait();
  uint32_t* const mine = peers[rank];
  __shared__ int ok, last;
  if (blockIdx.x == 0 && (int)threadIdx.x < world && (int)threadIdx.x != rank)
    st_release_sys(peers[threadIdx.x] + rank, epoch);
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = px_now_ns();
    for (int q = 0; q < world && ok; q++) {
      if (q == rank) continue;
      while (!px_reached(ld_acquire_sys(mine + q), epoch)) {
        if (px_now_ns() - t0 > kPxWaitNs) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) {
      atomicOr(status, ST_WAIT_TIMEOUT);
      atomicOr(mine + 129, 1u);
    }
  }
  __syncthreads();
  const long off = kPxFlagWords + (long)rank * words;
  const long nvec = words / 4;  // words is a multiple of 4 (the host checks)
  const uint4* src = reinterpret_cast<const uint4*>(mine + off);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; ok && i < nvec;
       i += (long)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    for (int q = 0; q < world; q++)
      if (q != rank) reinterpret_cast<uint4*>(peers[q] + off)[i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(mine + 128, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  mine[128] = 0;  // the ticket of the next call
  if (atomicExch(mine + 129, 0u) != 0u) return;  // a block's wait ran out: no done
  for (int q = 0; q < world; q++)
    if (q != rank) st_release_sys(peers[q] + 64 + rank, epoch);
  const uint64_t t0 = px_now_ns();
  for (int q = 0; q < world; q++) {
    if (q == rank) continue;
    while (!px_reached(ld_acquire_sys(mine + 64 + q), epoch)) {
      if (px_now_ns() - t0 > kPxWaitNs) {
        atomicOr(status, ST_WAIT_TIMEOUT);
        return;
      }
    }
  }
}

}  // namespace

void px_allgather(eb_engine* e, uint32_t* const* peers_d, int world, int rank, size_t words,
                  uint32_t epoch) {
  const size_t nvec = words / 4;
  const unsigned grid = (unsigned)std::min<size_t>(
      std::max<size_t>(1, (nvec + 255) / 256), (size_t)e->num_sms);
  launch_pdl(e, k_px_allgather, grid, 256, 0, peers_d, world, rank, (long)words, epoch,
             e->d_status);
  EB_LAUNCH("peer all-gather");
}

}  // namespace eb
