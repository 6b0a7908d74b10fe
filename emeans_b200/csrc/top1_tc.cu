// Exact top-1 on the tensor cores: a tcgen05 screen on 16-bit fixed-point
// operands held as two int8 digits, then the exact FP32 chain for the few
// centroids the screen cannot rule out. Top-k uses the same kernel and
// digits (k_screen<true, true>: the best kk screened values per row and the
// window below the kk-th); the internal scores' product uses it on split
// FP16 operands.
//
// The labels and scores are the reference CPU kernel's bit for bit
// (crates/emeans-core/src/assign/fused.rs:12-16: one sequential FMA chain per
// dot, lower id on ties). The screen only decides which centroids get that
// exact chain:
//
// 1. prep: each row is scaled by its own factor (the centroids by one) so
//    that its largest value is 32638, rounded to integers v, and kept as
//    digits v = 256 hi + lo (int8 each). A bound data set keeps this copy
//    across calls.
// 2. screen (tcgen05 kind::i8, persistent: one CTA per SM over 128-row
//    tiles): each 256-centroid tile accumulates hi.hi in one TMEM
//    accumulator and hi.lo + lo.hi in a second, both exact int32 sums;
//    operands arrive by TMA in 64-byte-swizzled shared memory through a
//    4-stage mbarrier ring. The epilogue (one thread per row) forms
//    hi.hi + floor((hi.lo + lo.hi) / 256) and converts it to FP32 once (in
//    units of 65536), tracks the running best
//    screened score and appends every centroid within 2e of it to the row's
//    candidate list, where e bounds |screen - exact chain|. A centroid more
//    than 2e behind the best cannot be the exact winner.
// 3. collect: each row's candidates still inside the final window become
//    (row, centroid) pairs.
// 4. pairs: one thread per pair runs the exact FMA chain (operands streamed
//    through shared memory) and folds (score, id) into the row's 64-bit key.
// 5. finish: labels and scores from the keys.
// 6. list: rows with non-finite inputs, too many candidates, or a screen that
//    gave up are scanned exactly against every centroid, parallel over
//    (row, block of centroids) with the same keyed reduction.
//
// Fixed-point error bound (integer units, x' and c' the scaled values): the
// rounding to integers, 0.502 sqrt(d) (|x'| + |c'|) + 0.252 d; the dropped
// lo.lo products, |x lo| |c lo|; the epilogue's evaluation, 65536 +
// 2^-22 (|x'| + 160 sqrt(d)) (|c'| + 160 sqrt(d)); and the FP32 chain,
// gamma_d |x'| |c'| (screen_bound_q8 derives each term).
//
// Split FP16 (the internal scores' products): values scaled by powers of two so that
// |v| < 2^14 and split into two FP16 terms, v' = hi + lo + r with
// |r| <= 2^-22 |v'| + 2^-24; its error bound in accumulator units (u = 2^-11):
//   split operands:   3 2^-22 sum|x'||c'| + 2^-23 (sum|x'| + sum|c'|)
//   accumulation:     d 2^-21 sum|x'||c'| (four times the per-addition
//                     truncation bound), the lo accumulator d 2^-30, the final
//                     add 2^-23
//   the FP32 chain:   gamma_d sum|x c| from the exact dot
// with sum|x'||c'| <= |x'| |c'| and sum|x'| <= sqrt(d) |x'| (Cauchy-Schwarz).
//
// Top-k mode holds the tile in TMEM while it scores: the best-kk state takes
// the registers that top-1 spends on the drained tile. It votes on each
// 16-column group first and scores in full only the groups that some row's
// window reaches, then releases the accumulators.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>

#include "engine.h"

namespace eb {

// The split FP16 screen copy of a bound data set, built by the first screened
// top-1 on the set and kept until the buffer is written or freed.
struct Fp16Copy {
  __half* xh = nullptr;  // n x dp, high terms
  __half* xl = nullptr;  // n x dp, low terms
  int* xexp = nullptr;
  float* xnrm = nullptr;
  size_t n = 0, d = 0;
  uint64_t version = 0;
  cudaStream_t stream = nullptr;
};

void free_copy(Fp16Copy* f) {
  if (!f) return;
  if (f->xh) cudaFreeAsync(f->xh, f->stream);
  if (f->xl) cudaFreeAsync(f->xl, f->stream);
  if (f->xexp) cudaFreeAsync(f->xexp, f->stream);
  if (f->xnrm) cudaFreeAsync(f->xnrm, f->stream);
  delete f;
}

// The fixed-point screen copy of a bound data set (top-1), built by the first
// top-1 on the set and kept like the split copy.
struct Q8Copy {
  int8_t* xh = nullptr;  // n x dp, high digits
  int8_t* xl = nullptr;  // n x dp, low digits
  float* xscl = nullptr;  // scales (0: not screened)
  float* xnrm = nullptr;
  float* xlo = nullptr;  // bounds on the low digits' norms
  size_t n = 0, d = 0;
  uint64_t version = 0;
  cudaStream_t stream = nullptr;
};

void free_q8(Q8Copy* f) {
  if (!f) return;
  for (void* p : {(void*)f->xh, (void*)f->xl, (void*)f->xscl, (void*)f->xnrm, (void*)f->xlo})
    if (p) cudaFreeAsync(p, f->stream);
  delete f;
}

void drop_f16(eb_buf* b) {
  if (b && b->f16) {
    free_copy(b->f16);
    b->f16 = nullptr;
  }
  if (b && b->q8) {
    free_q8(b->q8);
    b->q8 = nullptr;
  }
}

namespace {

constexpr int BM = 128;          // rows per tile (TMEM lanes)
constexpr int BN = 256;          // centroids per tile (TMEM columns per accumulator)
constexpr int BKH = 32;          // FP16 columns per k-block: one 64-byte swizzle row
constexpr int BK8 = 64;          // int8 columns per k-block (top-1): the same 64 bytes
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKH * 2;                // one of xh / xl
constexpr int B_BYTES = BN * BKH * 2;                // one of ch / cl
constexpr int STAGE_BYTES = 2 * (A_BYTES + B_BYTES);
constexpr int CAP = 64;          // per-row candidate list capacity
constexpr int CAP_TOPK = 128;    // the same in top-k mode (lists there grow further)
constexpr int SURV = 64;         // candidates per row taken to exact chains (more: full scan)
constexpr int KMAX = 16;         // largest k of the top-k mode
// Three warpgroups: warp 0 TMA, warp 1 MMA (warps 2-3 idle), warps 4-11 epilogue.
// Launched at 168 registers a thread; the first warpgroup gives its registers
// to the epilogue (setmaxnreg: 128 x 56 + 256 x 224 = 384 x 168).
constexpr int NTHREADS = 384;
constexpr int REG_PRODUCER = 56, REG_EPILOGUE = 224;
static_assert(128 * REG_PRODUCER + 256 * REG_EPILOGUE <= NTHREADS * 168, "register split");
constexpr int HALF = BN / 2;     // tile columns per epilogue warp (two warps per TMEM lane quadrant)
constexpr uint32_t FALLBACK = 0xFFFFFFFFu;
constexpr int XEXP_BAD = INT_MIN;  // row with a non-finite value
constexpr size_t PASS_WAVES = 8;   // row tiles per SM in one pass (top-k, products)
constexpr size_t PASS_WAVES_TOP1 = 12;  // at most, in one top-1 pass
constexpr uint64_t WAIT_NS = 2000000000ull;  // bounded waits: 2 s

// Operand ring, 256 B of barriers / TMEM slot / flags, the centroid norms of
// each epilogue warp's half tile, and each epilogue warp's slab of one
// group's screened values ([16 columns][32 rows]) for the appends.
constexpr size_t SMEM_BYTES = 1024 /* alignment slack */ + STAGES * STAGE_BYTES + 256 +
                              8 * HALF * sizeof(float) + 8 * 16 * 32 * sizeof(float);

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `bar` with the given parity; false (and the CTA's
// abort flag set) after WAIT_NS, so that no wait can spin forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (now_ns() - t0 > WAIT_NS) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// K-major operand tile with 64-byte rows, 64B swizzle, 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;   // stride byte offset: 8 rows x 64 B
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;            // SWIZZLE_64B
  return d;
}

// kind::f16 instruction descriptor: F16 x F16 -> F32, both K-major, M=128, N=256.
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
      : "memory");
}

// kind::i8 instruction descriptor: S8 x S8 -> S32, both K-major, M=128, N=256.
constexpr uint32_t IDESC_I8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                              ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC_I8), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 16 consecutive FP32 columns of this thread's TMEM lane (valid after
// tmem_wait_tied()).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// An empty statement that takes registers loaded from TMEM as operands: placed
// after tmem_wait(), it keeps the compiler from moving their uses above it.
__device__ __forceinline__ void tmem_tie(uint32_t (&a)[16]) {
  asm volatile(""
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                 "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]),
                 "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]));
}
// Keep only the entries of a row's candidate list still inside the window
// (out of line: it runs only when a list nears its capacity). Entries are
// read eight at a time before any of them is written back: every write goes
// to a slot at or below one already read, so the batch's loads can all be in
// flight together.
template <bool IP>
__device__ __noinline__ uint32_t compact_list(uint2* list, long stride, uint32_t cnt, float thr) {
  uint32_t w = 0;
  for (uint32_t e0 = 0; e0 < cnt; e0 += 8) {
    uint2 en[8];
#pragma unroll
    for (int u = 0; u < 8; u++)
      en[u] = e0 + u < cnt ? list[(e0 + u) * stride] : make_uint2(0u, __float_as_uint(NAN));
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const float sv = __uint_as_float(en[u].y);
      if (IP ? (sv >= thr) : (sv <= thr)) list[(w++) * stride] = en[u];
    }
  }
  return w;
}

// ---------------------------------------------------------------- prep kernels

// Split a scaled value into two FP16 terms: hi = RN(v), lo = RN(v - hi); the
// difference v - hi is exact in FP32.
__device__ __forceinline__ void split16(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

// Scaled split FP16 copy of the selected rows (one warp per row), with the
// row's exponent (XEXP_BAD for non-finite rows) and an upper bound on its norm.
__global__ void k_prep_rows(const float* __restrict__ x, long n, int d, int dp,
                            const uint32_t* __restrict__ ids, long p0, long m,
                            __half* __restrict__ xh, __half* __restrict__ xl,
                            int* __restrict__ xexp, float* __restrict__ xnrm, uint32_t* status) {
  pdl_wait();
  const long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= m) return;
  const long p = p0 + i;
  const long row = ids ? (long)ids[p] : p;
  __half* oh = xh + i * (long)dp;
  __half* ol = xl + i * (long)dp;
  if (row >= n) {
    if (lane == 0) {
      atomicOr(status, ST_BAD_ROW);
      xexp[i] = XEXP_BAD;
      xnrm[i] = 0.0f;
    }
    for (int t = lane; t < dp; t += 32) oh[t] = ol[t] = __float2half_rn(0.0f);
    return;
  }
  const float* r = x + row * (long)d;
  float mx = 0.0f, ss = 0.0f;
  bool finite = true;
  int ex = 0;
  if ((d & 3) == 0 && d <= 1024) {
    // One read: up to 8 float4 per lane stay in registers.
    const float4* r4 = reinterpret_cast<const float4*>(r);
    const int q4 = d / 4;
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int t = lane + 32 * u;
      v[u] = t < q4 ? __ldg(r4 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
      finite = finite && isfinite(v[u].x) && isfinite(v[u].y) && isfinite(v[u].z) &&
               isfinite(v[u].w);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
      ss = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, fmaf(v[u].w, v[u].w, ss))));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    }
    finite = __all_sync(0xFFFFFFFFu, finite);
    frexpf(mx, &ex);
    const int sh = 14 - ex;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int t = lane + 32 * u;
      if (t < q4) {
        const float a[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        __half h[4], l[4];
#pragma unroll
        for (int w = 0; w < 4; w++) split16(finite ? ldexpf(a[w], sh) : 0.0f, h[w], l[w]);
        __half2 h01 = __halves2half2(h[0], h[1]), h23 = __halves2half2(h[2], h[3]);
        __half2 l01 = __halves2half2(l[0], l[1]), l23 = __halves2half2(l[2], l[3]);
        *reinterpret_cast<uint2*>(oh + 4 * t) =
            make_uint2(*reinterpret_cast<uint32_t*>(&h01), *reinterpret_cast<uint32_t*>(&h23));
        *reinterpret_cast<uint2*>(ol + 4 * t) =
            make_uint2(*reinterpret_cast<uint32_t*>(&l01), *reinterpret_cast<uint32_t*>(&l23));
      }
    }
    for (int t = d + lane; t < dp; t += 32) oh[t] = ol[t] = __float2half_rn(0.0f);
  } else {
    for (int t = lane; t < d; t += 32) {
      const float v = __ldg(r + t);
      finite = finite && isfinite(v);
      mx = fmaxf(mx, fabsf(v));
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    }
    finite = __all_sync(0xFFFFFFFFu, finite);
    frexpf(mx, &ex);
    const int sh = 14 - ex;
    for (int t = lane; t < dp; t += 32) {
      const float v = t < d ? __ldg(r + t) : 0.0f;
      split16(finite ? ldexpf(v, sh) : 0.0f, oh[t], ol[t]);
    }
  }
  if (lane == 0) {
    xexp[i] = finite ? ex : XEXP_BAD;
    // Any-order sum of squares: relative error < d 2^-24; inflate by 2^-9.
    xnrm[i] = finite ? sqrtf(ss) * (1.0f + 1.0f / 512.0f) : 0.0f;
  }
}

// ---- the top-1 screen's fixed-point copies
//
// A row (or the centroid set) is scaled by s = 32638 / max |x| (FP32, so
// that the largest scaled value rounds to at most 32638.01), and each value
// rounded to the integer v = rint(fl(x s)) (|x s - v| <= 1/2 + 2^-24 32639
// < 0.502), kept as two int8 digits v = 256 hi + lo, hi in [-127, 127], lo
// in [-128, 127].

// The scale of a set with largest magnitude mx (1 for mx = 0; not finite
// when mx is too small for 32638 / mx).
__device__ __forceinline__ float q8_scale(float mx) {
  return mx > 0.0f ? __fdiv_rn(32638.0f, mx) : 1.0f;
}

// The digits of an integral v with |v| <= 32639 = 256 x 127 + 127 (every
// step exact).
__device__ __forceinline__ void split8(float v, int& hi, int& lo) {
  hi = __float2int_rd((v + 128.0f) * (1.0f / 256.0f));
  lo = (int)v - 256 * hi;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | (uint32_t)(b & 0xFF) << 8 | (uint32_t)(c & 0xFF) << 16 |
         (uint32_t)(d & 0xFF) << 24;
}

// Fixed-point copy of the selected rows (one warp per row): digits xh, xl
// (dp bytes a row, zero-padded), the row's scale (0 for rows with a
// non-finite value or no finite scale), an upper bound on its norm and on
// the norm of its low digits.
__global__ void k_prep_rows_q8(const float* __restrict__ x, long n, int d, int dp,
                               const uint32_t* __restrict__ ids, long p0, long m,
                               int8_t* __restrict__ xh, int8_t* __restrict__ xl,
                               float* __restrict__ xscl, float* __restrict__ xnrm,
                               float* __restrict__ xlo, uint32_t* status) {
  pdl_wait();
  const long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= m) return;
  const long p = p0 + i;
  const long row = ids ? (long)ids[p] : p;
  int8_t* oh = xh + i * (long)dp;
  int8_t* ol = xl + i * (long)dp;
  if (row >= n) {
    if (lane == 0) {
      atomicOr(status, ST_BAD_ROW);
      xscl[i] = 0.0f;
      xnrm[i] = 0.0f;
      xlo[i] = 0.0f;
    }
    for (int t = lane; t < dp / 4; t += 32)
      reinterpret_cast<uint32_t*>(oh)[t] = reinterpret_cast<uint32_t*>(ol)[t] = 0u;
    return;
  }
  const float* r = x + row * (long)d;
  float mx = 0.0f, ss = 0.0f, sl = 0.0f;
  bool finite = true;
  float sc = 1.0f;
  if ((d & 3) == 0 && d <= 1024) {
    // One read: up to 8 float4 per lane stay in registers.
    const float4* r4 = reinterpret_cast<const float4*>(r);
    const int q4 = d / 4;
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int t = lane + 32 * u;
      v[u] = t < q4 ? __ldg(r4 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
      finite = finite && isfinite(v[u].x) && isfinite(v[u].y) && isfinite(v[u].z) &&
               isfinite(v[u].w);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
      ss = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, fmaf(v[u].w, v[u].w, ss))));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    }
    finite = __all_sync(0xFFFFFFFFu, finite);
    sc = q8_scale(mx);
    finite = finite && isfinite(sc);
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int t = lane + 32 * u;
      if (t < q4) {
        const float a[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        int h[4], l[4];
#pragma unroll
        for (int w = 0; w < 4; w++) {
          split8(finite ? rintf(__fmul_rn(a[w], sc)) : 0.0f, h[w], l[w]);
          sl = fmaf((float)l[w], (float)l[w], sl);
        }
        reinterpret_cast<uint32_t*>(oh)[t] = pack4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<uint32_t*>(ol)[t] = pack4(l[0], l[1], l[2], l[3]);
      }
    }
    for (int t = q4 + lane; t < dp / 4; t += 32)
      reinterpret_cast<uint32_t*>(oh)[t] = reinterpret_cast<uint32_t*>(ol)[t] = 0u;
  } else {
    for (int t = lane; t < d; t += 32) {
      const float v = __ldg(r + t);
      finite = finite && isfinite(v);
      mx = fmaxf(mx, fabsf(v));
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    }
    finite = __all_sync(0xFFFFFFFFu, finite);
    sc = q8_scale(mx);
    finite = finite && isfinite(sc);
    for (int t = lane; t < dp; t += 32) {
      const float v = (t < d && finite) ? rintf(__fmul_rn(__ldg(r + t), sc)) : 0.0f;
      int h, l;
      split8(v, h, l);
      oh[t] = (int8_t)h;
      ol[t] = (int8_t)l;
      sl = fmaf((float)l, (float)l, sl);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) sl += __shfl_xor_sync(0xFFFFFFFFu, sl, o);
  if (lane == 0) {
    xscl[i] = finite ? sc : 0.0f;
    // Any-order sums of squares: relative error < d 2^-24; inflate by 2^-9.
    xnrm[i] = finite ? sqrtf(ss) * (1.0f + 1.0f / 512.0f) : 0.0f;
    xlo[i] = finite ? sqrtf(sl) * (1.0f + 1.0f / 512.0f) : 0.0f;
  }
}

// Rows x[ids[p]] of a cached fixed-point copy gathered into the pass's
// staging rows (one warp per row, 16-byte copies; dp is a multiple of 64).
__global__ void k_gather_rows_q8(const int8_t* __restrict__ src_h, const int8_t* __restrict__ src_l,
                                 const float* __restrict__ src_s, const float* __restrict__ src_n,
                                 const float* __restrict__ src_lo, long n, int dp,
                                 const uint32_t* __restrict__ ids, long p0, long m,
                                 int8_t* __restrict__ xh, int8_t* __restrict__ xl,
                                 float* __restrict__ xscl, float* __restrict__ xnrm,
                                 float* __restrict__ xlo, uint32_t* status) {
  pdl_wait();
  const long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= m) return;
  const long row = ids[p0 + i];
  uint4* oh = reinterpret_cast<uint4*>(xh + i * (long)dp);
  uint4* ol = reinterpret_cast<uint4*>(xl + i * (long)dp);
  const int q = dp / 16;
  if (row >= n) {
    for (int t = lane; t < q; t += 32) oh[t] = ol[t] = make_uint4(0, 0, 0, 0);
    if (lane == 0) {
      atomicOr(status, ST_BAD_ROW);
      xscl[i] = 0.0f;
      xnrm[i] = 0.0f;
      xlo[i] = 0.0f;
    }
    return;
  }
  const uint4* ih = reinterpret_cast<const uint4*>(src_h + row * (long)dp);
  const uint4* il = reinterpret_cast<const uint4*>(src_l + row * (long)dp);
  for (int t = lane; t < q; t += 32) {
    oh[t] = __ldg(ih + t);
    ol[t] = __ldg(il + t);
  }
  if (lane == 0) {
    xscl[i] = src_s[row];
    xnrm[i] = src_n[row];
    xlo[i] = src_lo[row];
  }
}

// The centroid summary: u64 words (generation << 32 | payload), [0] bits of
// max |c|, [1] bits of a bound on max |c_j|, [2] non-finite flag, [3] (the
// fixed-point conversion) bits of a bound on the largest norm of a
// centroid's low digits. The words
// are atomic maxima, so a word from an older generation (a smaller tag) is
// replaced by the first write of this one; a reader takes a word whose tag is
// not the current generation as 0.
__device__ __forceinline__ uint32_t cinfo_word(const unsigned long long* ci, int w, uint32_t gen) {
  const unsigned long long v = ci[w];
  return (uint32_t)(v >> 32) == gen ? (uint32_t)v : 0u;
}

// Global max |c|, a bound on max |c_j| and a non-finite flag, over all
// centroids, into the summary of generation gen. One warp per centroid, two
// per block; 16-byte loads when the rows allow.
__global__ void __launch_bounds__(64) k_cent_max(const float* __restrict__ c, long k, int d,
                                                 unsigned long long* cinfo, uint32_t gen) {
  pdl_wait();
  const long j = (long)blockIdx.x * 2 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (j >= k) return;
  const float* r = c + j * (long)d;
  float mx = 0.0f, ss = 0.0f;
  bool finite = true;
  if ((d & 3) == 0 && ((uintptr_t)c & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(r);
#pragma unroll 4
    for (int t = lane; t < d / 4; t += 32) {
      const float4 v = __ldg(r4 + t);
      finite = finite && isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
  } else {
    for (int t = lane; t < d; t += 32) {
      const float v = __ldg(r + t);
      finite = finite && isfinite(v);
      mx = fmaxf(mx, fabsf(v));
      ss = fmaf(v, v, ss);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  }
  finite = __all_sync(0xFFFFFFFFu, finite);
  if (lane == 0) {
    const unsigned long long tag = (unsigned long long)gen << 32;
    if (!finite) {
      summary_max(&cinfo[2], tag | 1ull);
      return;
    }
    summary_max(&cinfo[0], tag | __float_as_uint(mx));
    summary_max(&cinfo[1], tag | __float_as_uint(sqrtf(ss) * (1.0f + 1.0f / 512.0f)));
  }
}

// Scaled split FP16 centroids: c' = c 2^(14 - ec), 2^(ec-1) <= max|c| < 2^ec.
// One warp per centroid, two per block; four columns per lane step when the
// rows allow 16-byte loads (dp is a multiple of 32, so the padding is whole
// groups of four).
__global__ void __launch_bounds__(64) k_cent_conv(const float* __restrict__ c, long k, int d,
                                                  int dp,
                                                  const unsigned long long* __restrict__ cinfo,
                                                  uint32_t gen, __half* __restrict__ ch,
                                                  __half* __restrict__ cl) {
  pdl_wait();
  const long j = (long)blockIdx.x * 2 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (j >= k) return;
  int ec = 0;
  frexpf(__uint_as_float(cinfo_word(cinfo, 0, gen)), &ec);
  const int sh = 14 - ec;
  const bool bad = cinfo_word(cinfo, 2, gen) != 0;
  const float* r = c + j * (long)d;
  __half* oh = ch + j * (long)dp;
  __half* ol = cl + j * (long)dp;
  if ((d & 3) == 0 && ((uintptr_t)c & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(r);
#pragma unroll 2
    for (int t = lane; t < dp / 4; t += 32) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (4 * t < d && !bad) v = __ldg(r4 + t);
      __align__(8) __half h[4], l[4];
      split16(ldexpf(v.x, sh), h[0], l[0]);
      split16(ldexpf(v.y, sh), h[1], l[1]);
      split16(ldexpf(v.z, sh), h[2], l[2]);
      split16(ldexpf(v.w, sh), h[3], l[3]);
      *reinterpret_cast<uint2*>(oh + 4 * t) = *reinterpret_cast<const uint2*>(h);
      *reinterpret_cast<uint2*>(ol + 4 * t) = *reinterpret_cast<const uint2*>(l);
    }
  } else {
    for (int t = lane; t < dp; t += 32) {
      const float v = (t < d && !bad) ? __ldg(r + t) : 0.0f;
      split16(ldexpf(v, sh), oh[t], ol[t]);
    }
  }
}

// Fixed-point centroids under the set's one scale (from max |c|): digits ch,
// cl (dp bytes a centroid, zero-padded), and the largest norm of a centroid's
// low digits into summary word 3. One warp per centroid, two per block.
__global__ void __launch_bounds__(64) k_cent_conv_q8(const float* __restrict__ c, long k, int d,
                                                     int dp,
                                                     unsigned long long* __restrict__ cinfo,
                                                     uint32_t gen, int8_t* __restrict__ ch,
                                                     int8_t* __restrict__ cl) {
  pdl_wait();
  const long j = (long)blockIdx.x * 2 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (j >= k) return;
  const float sc = q8_scale(__uint_as_float(cinfo_word(cinfo, 0, gen)));
  const bool bad = cinfo_word(cinfo, 2, gen) != 0 || !isfinite(sc);
  const float* r = c + j * (long)d;
  int8_t* oh = ch + j * (long)dp;
  int8_t* ol = cl + j * (long)dp;
  float sl = 0.0f;
  if ((d & 3) == 0 && ((uintptr_t)c & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(r);
#pragma unroll 2
    for (int t = lane; t < dp / 4; t += 32) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (4 * t < d && !bad) v = __ldg(r4 + t);
      const float a[4] = {v.x, v.y, v.z, v.w};
      int h[4], l[4];
#pragma unroll
      for (int w = 0; w < 4; w++) {
        split8(rintf(__fmul_rn(a[w], sc)), h[w], l[w]);
        sl = fmaf((float)l[w], (float)l[w], sl);
      }
      reinterpret_cast<uint32_t*>(oh)[t] = pack4(h[0], h[1], h[2], h[3]);
      reinterpret_cast<uint32_t*>(ol)[t] = pack4(l[0], l[1], l[2], l[3]);
    }
  } else {
    for (int t = lane; t < dp; t += 32) {
      const float v = (t < d && !bad) ? rintf(__fmul_rn(__ldg(r + t), sc)) : 0.0f;
      int h, l;
      split8(v, h, l);
      oh[t] = (int8_t)h;
      ol[t] = (int8_t)l;
      sl = fmaf((float)l, (float)l, sl);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) sl += __shfl_xor_sync(0xFFFFFFFFu, sl, o);
  if (lane == 0)
    summary_max(&cinfo[3], (unsigned long long)gen << 32 |
                             __float_as_uint(sqrtf(sl) * (1.0f + 1.0f / 512.0f)));
}

// Top-k mode: v (> kv[0]) replaces the smallest of the ascending kv[0 .. KMAX)
// and takes its place in the order. The slots below v's place each take the
// next slot's value: independent selects instead of a chain of KMAX - 1
// compare-exchanges.
__device__ __forceinline__ void kv_insert(float (&kv)[KMAX], float v) {
  float nk[KMAX];
#pragma unroll
  for (int a = 0; a < KMAX; a++) {
    const bool shift = a + 1 < KMAX && kv[a + 1] < v;          // a is below v's place
    const bool here = !shift && (a == 0 || kv[a] < v);           // v's place
    nk[a] = shift ? kv[a + 1] : (here ? v : kv[a]);
  }
#pragma unroll
  for (int a = 0; a < KMAX; a++) kv[a] = nk[a];
}

// ---------------------------------------------------------------- the screen

struct ScreenParams {
  long m;              // staging rows in this pass
  int k;
  int kblocks;         // dp / 32
  int ntiles;          // ceil(k / 256)
  // Work units: (row tile, part) pairs, unit u = row tile u / parts, part
  // u % parts, which covers centroid tiles part * tpp .. min(+ tpp, ntiles).
  // Splitting a row tile's centroid tiles over parts fills the SMs when there
  // are few row tiles (a training batch's slice on one of several GPUs).
  int parts;
  int tpp;             // centroid tiles per part
  int units;           // ceil(m / 128) * parts
  const int* xexp;     // per staging row (split FP16)
  const float* xscl;   // per staging row (fixed point: the row's scale, 0 = not screened)
  const float* xnrm;   // per staging row
  const float* xlo;    // per staging row, fixed point: a bound on its low digits' norm
  const float* cn;     // k squared centroid norms (L2) or null
  const unsigned long long* cinfo;  // the centroid summary of generation cgen
  uint32_t cgen;
  float e_rel, e_abs, e_min;  // bound coefficients (see the header comment)
  float e_lo;                 // fixed point: the coefficient of the low-digit term
  // Candidate lists, one per (part, half tile, row): list L = 2 part + half,
  // entry e of row i at (L C + e) m + i (id, screened value bits), C = CAP
  // (CAP_TOPK in top-k mode; top-k mode has one part).
  uint2* cand;
  uint32_t* cand_cnt;  // 2 parts m: entries in use per (list, row), or FALLBACK
  float* cand_thr;     // 2 parts m: the final admission threshold per (list, row)
  uint32_t* status;
  // Top-k mode (k_screen<true, true>): each (row, half) keeps its best kk
  // screened values and admits every column within the window of the kk-th.
  int kk;
  int exclude_self;    // skip the column whose id is the row's global id
  long row_gid0;       // global id of staging row 0
  long col_gid0;       // global id of column 0 (a database shard's offset)
  float* kvals;        // 2 m x KMAX: each (half, row)'s best kk values, ascending
  float* roff;         // m: each row's window 2e
  // Counters of the exact stage that follows (pairs, exact list), zeroed by
  // the screen's first thread.
  uint32_t* zero0;
  uint32_t* zero1;
  // Product mode (k_screen<true, false, true>, the internal scores' n x k
  // product): each row's own column pslot[plabels[prow0 + i]], per column the
  // weight pinv (1 / cluster size), and per (list, row) the largest weighted
  // product over the other columns (pmax, in accumulator units) and its
  // column (pcol; the lower column on ties).
  const uint32_t* plabels;
  const uint32_t* pslot;
  long prow0;
  const float* pinv;
  float* pmax;
  uint32_t* pcol;
  // Failure-detection test (eb_test_screen_dead_wait): CTA 0's epilogue waits
  // for its second tile on a barrier that nothing arrives at, so that the
  // wait runs out and the give-up path runs. 0 in normal use.
  int dead_wait;
};

template <bool IP, bool TOPK = false, bool PROD = false, bool Q8 = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_screen(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
             const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
             ScreenParams P) {
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 1;
  uint64_t* mma_done = tempty + 1;
  uint64_t* dead = mma_done + 1;  // never arrived at (the dead_wait test)
  uint32_t* tmem_slot = (uint32_t*)(dead + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* cn_s = (float*)(smem + STAGES * STAGE_BYTES + 256);  // [8 warps][HALF]
  float* sv_s = cn_s + 8 * HALF;                               // [8 warps][16][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Top-k runs on the fixed-point digits only (the split FP16 operands serve
  // the product mode).
  static_assert(!TOPK || Q8, "top-k mode reads fixed-point digits");

  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      if (P.zero0) *P.zero0 = 0u;
      if (P.zero1) *P.zero1 = 0u;
    }
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 256);
    mbar_init(mma_done, 1);
    mbar_init(dead, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // hi accumulator at column 0, lo at column BN
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PRODUCER));
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: per (row tile, centroid tile, k-block) the four boxes
      // xh, xl (128 x 32) and ch, cl (256 x 32). The ring runs on across tiles.
      int it = 0, issued = 0;
      bool stop = false;
      for (int u = blockIdx.x; u < P.units && !stop; u += gridDim.x) {
        const int rt = u / P.parts;
        const int nt0 = (u % P.parts) * P.tpp, nt1 = min(nt0 + P.tpp, P.ntiles);
        for (int t2 = nt0 * P.kblocks; t2 < nt1 * P.kblocks; t2++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag)) {
            stop = true;
            break;
          }
          const int nt = t2 / P.kblocks, kb = t2 % P.kblocks;
          uint8_t* st = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          const int kx = kb * (Q8 ? BK8 : BKH);  // 64 bytes of every row either way
          tma_load_2d(st, &tmAh, &full[s], kx, (int)(rt * BM));
          tma_load_2d(st + A_BYTES, &tmAl, &full[s], kx, (int)(rt * BM));
          tma_load_2d(st + 2 * A_BYTES, &tmBh, &full[s], kx, nt * BN);
          tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tmBl, &full[s], kx, nt * BN);
          issued = it + 1;
        }
      }
      // No copy may still be landing in shared memory when the CTA exits: wait
      // (bounded) for the last loads issued. On the normal path they have
      // already been consumed and these waits return at once.
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; j++) {
        const uint64_t t0 = now_ns();
        while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && now_ns() - t0 < WAIT_NS) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer; tc counts (row tile, centroid tile) pairs.
      int it = 0, tc = 0;
      bool stop = false;
      for (int u = blockIdx.x; u < P.units && !stop; u += gridDim.x) {
        const int nt0 = (u % P.parts) * P.tpp, nt1 = min(nt0 + P.tpp, P.ntiles);
        for (int nt = nt0; nt < nt1; nt++, tc++) {
          // The epilogue must have read both accumulators of the last tile.
          if (!mbar_wait(tempty, (tc & 1) ^ 1, abort_flag)) {
            stop = true;
            break;
          }
          tc_fence_after();
          bool ok = true;
          for (int kb = 0; kb < P.kblocks; kb++, it++) {
            const int s = it % STAGES;
            if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ah = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t al = ah + A_BYTES, bh = ah + 2 * A_BYTES, bl = bh + B_BYTES;
#pragma unroll
            for (int kk = 0; kk < BKH / 16; kk++) {
              const uint32_t first = (kb > 0 || kk > 0) ? 1u : 0u;
              if constexpr (Q8) {
                // 32 int8 columns per MMA: hi.hi, and hi.lo + lo.hi (exact int32 sums).
                umma_i8(tmem, umma_desc(ah + kk * 32), umma_desc(bh + kk * 32), first);
                umma_i8(tmem + BN, umma_desc(ah + kk * 32), umma_desc(bl + kk * 32), first);
                umma_i8(tmem + BN, umma_desc(al + kk * 32), umma_desc(bh + kk * 32), 1u);
              } else {
                umma_f16(tmem, umma_desc(ah + kk * 32), umma_desc(bh + kk * 32), first);
                umma_f16(tmem + BN, umma_desc(ah + kk * 32), umma_desc(bl + kk * 32), first);
                umma_f16(tmem + BN, umma_desc(al + kk * 32), umma_desc(bh + kk * 32), 1u);
              }
            }
            umma_commit(&empty[s]);
          }
          if (!ok) {
            stop = true;
            break;
          }
          umma_commit(tfull);
        }
      }
      // Every MMA this thread issued has completed once mma_done flips.
      umma_commit(mma_done);
      const uint64_t t0 = now_ns();
      while (!mbar_try_wait(mma_done, 0) && now_ns() - t0 < WAIT_NS) {
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPILOGUE));
    // Epilogue: warps 4-11. Warp w reads TMEM lanes 32 (w % 4) .. + 31 (one
    // row per thread) and half (w - 4) / 4 of every tile's columns; each
    // (row, half) keeps its own running best and candidate list.
    const int q = warp & 3;
    const int hf = (warp - 4) >> 2;
    const int r = q * 32 + lane;
    // The centroids' scale: split FP16, c' = c 2^(14 - ec); fixed point,
    // c' = c csc, and a bound on their low digits' norms.
    int ec = 0;
    float csc = 1.0f;
    if constexpr (Q8)
      csc = q8_scale(__uint_as_float(cinfo_word(P.cinfo, 0, P.cgen)));
    else
      frexpf(__uint_as_float(cinfo_word(P.cinfo, 0, P.cgen)), &ec);
    const float cmax = __uint_as_float(cinfo_word(P.cinfo, 1, P.cgen));
    const bool c_bad = cinfo_word(P.cinfo, 2, P.cgen) != 0 || !isfinite(csc);
    const float clo = Q8 ? __uint_as_float(cinfo_word(P.cinfo, 3, P.cgen)) : 0.0f;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(hf * HALF);
    float* cns = cn_s + (warp - 4) * HALF;
    float* svs = sv_s + (warp - 4) * 16 * 32 + lane;  // this lane's column of the slab
    int tc = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < P.units; u += gridDim.x) {
      const long rt = u / P.parts;
      const int part = u % P.parts;
      const int nt0 = part * P.tpp, nt1 = min(nt0 + P.tpp, P.ntiles);
      const int L = 2 * part + hf;  // this (part, half)'s candidate list
      const long i = rt * BM + r;
      const bool live = i < P.m;
      if (stop) {
        // A wait gave up: this CTA's remaining rows go to the exact fallback
        // (product mode: no result; the call reports the timeout).
        if (live) {
          if (PROD)
            P.pmax[L * P.m + i] = NAN;
          else
            P.cand_cnt[L * P.m + i] = FALLBACK;
        }
        continue;
      }
      const int ex = live && !Q8 ? P.xexp[i] : XEXP_BAD;
      const float xsc = live && Q8 ? P.xscl[i] : 0.0f;
      bool fallback = !live || c_bad || (Q8 ? !(xsc > 0.0f) : ex == XEXP_BAD);
      const float xn = live ? P.xnrm[i] : 0.0f;
      // |x'| and max |c'| in accumulator units, and the bound e there. Fixed
      // point: x' = x xsc, c' = c csc, and the dropped lo.lo products add at
      // most |x lo| max |c lo|.
      const float xs = Q8 ? xn * (fallback ? 1.0f : xsc) : ldexpf(xn, 14 - (fallback ? 0 : ex));
      const float cs = Q8 ? cmax * csc : ldexpf(cmax, 14 - ec);
      float e_acc = fmaf(P.e_rel * xs, cs, fmaf(P.e_abs, xs + cs, P.e_min));
      // Fixed point: the accumulator value is in units of 65536 (hi.hi).
      if (Q8) e_acc = fmaf(P.e_lo * (live ? P.xlo[i] : 0.0f), clo, e_acc) * (1.0f / 65536.0f);
      float off, m2f = 1.0f;  // screened value = m2f acc + cn (IP: acc + 0)
      if (IP) {
        off = 2.0f * e_acc;
      } else {
        // The dot is f acc: 2^(ex + ec - 28), or 1 / (xsc csc) rounded (its
        // relative error 2^-22 is a third rounding of the key's dot term).
        float f;
        if constexpr (Q8) {
          f = fallback ? 1.0f : __frcp_rn(__fmul_rn(xsc, csc)) * 65536.0f;
          if (!(f > 0.0f) || !isfinite(f)) fallback = true;
        } else {
          const int fe = ex + ec - 28;
          if (fe < -100 || fe > 100) fallback = true;
          f = ldexpf(1.0f, fallback ? 0 : fe);
        }
        m2f = -2.0f * f;
        // key error: twice the dot error plus the key's roundings.
        const float e_key =
            fmaf(2.0f * f, e_acc, ldexpf(fmaf(cmax, cmax, 2.0f * xn * cmax), Q8 ? -21 : -22));
        off = 2.0f * e_key;
      }
      if (!isfinite(off)) fallback = true;
      const bool collect = live && !fallback;
      // Product mode: this row's own column and the running maximum.
      const long own_col = PROD && live ? (long)P.pslot[P.plabels[P.prow0 + i]] : -1;
      float pm = -INFINITY;
      uint32_t pc = 0xFFFFFFFFu;
      float best = IP ? -INFINITY : INFINITY;
      float thr = best;
      bool overflow = false;
      uint32_t cnt = 0;  // entries in this (row, half)'s candidate list
      constexpr int LCAP = TOPK ? CAP_TOPK : CAP;
      uint2* row_list = P.cand + (long)L * LCAP * P.m + (live ? i : 0);  // entries P.m apart
      // Top-k mode: the best kk screened values so far in slots 0 .. kk - 1,
      // ascending (the kk-th best in slot 0), slots kk .. KMAX - 1 held at +inf.
      float kv[TOPK ? KMAX : 1];
#pragma unroll
      for (int a = 0; a < (TOPK ? KMAX : 1); a++) kv[a] = a < P.kk ? -INFINITY : INFINITY;
      float kth = -INFINITY;
      const long gid = P.row_gid0 + i;

      for (int nt = nt0; nt < nt1; nt++, tc++) {
        // Warp-uniform: the TMEM loads below are .sync.aligned.
        uint64_t* wbar = tfull;
        uint32_t wpar = tc & 1;
        const int col0 = nt * BN + hf * HALF;  // first centroid of this warp's half tile
        // This half tile's squared centroid norms (product mode: the columns'
        // weights), loaded before the wait for the accumulators so that their
        // latency overlaps the MMAs, and staged in the warp's own shared
        // memory after the drain (no barrier across warps, so a timed-out
        // wait strands no warp).
        float cnv[HALF / 32];
        if (!IP || PROD) {
          const float* src = PROD ? P.pinv : P.cn;
#pragma unroll
          for (int u = 0; u < HALF / 32; u++) {
            const int c = u * 32 + lane;
            cnv[u] = col0 + c < P.k ? __ldg(src + col0 + c) : 0.0f;
          }
        }
        if (P.dead_wait && blockIdx.x == 0 && tc == 1) {
          wbar = dead;  // phase 0 never completes: the wait runs out after WAIT_NS
          wpar = 0;
        }
        const bool ready = __all_sync(0xFFFFFFFFu, mbar_wait(wbar, wpar, abort_flag));
        if (!ready) {
          stop = true;
          break;
        }
        tc_fence_after();
        const int ngr = max(0, min(HALF / 16, (P.k - col0 + 15) / 16));
        // Drain: this thread's half-tile row (hi in acc, lo added group pair by
        // group pair) comes into registers and the accumulators are released
        // at once, so that the next tile's products run while this one is
        // scored.
        constexpr int LOG = 2;  // lo groups per TMEM wait
        uint32_t acc[TOPK ? 1 : HALF / 16][16];
        if constexpr (!TOPK) {
          uint32_t lo[LOG][16];
#pragma unroll
          for (int g = 0; g < HALF / 16; g++)
            if (g < ngr) tmem_ld16(lane_base + (uint32_t)(g * 16), acc[g]);
#pragma unroll
          for (int p2 = 0; p2 < HALF / 16 / LOG; p2++) {
#pragma unroll
            for (int h2 = 0; h2 < LOG; h2++)
              if (LOG * p2 + h2 < ngr)
                tmem_ld16(lane_base + (uint32_t)(BN + (LOG * p2 + h2) * 16), lo[h2]);
            tmem_wait();
            if (p2 == 0) {
#pragma unroll
              for (int g = 0; g < HALF / 16; g++) tmem_tie(acc[g]);
            }
#pragma unroll
            for (int h2 = 0; h2 < LOG; h2++) tmem_tie(lo[h2]);
#pragma unroll
            for (int h2 = 0; h2 < LOG; h2++)
#pragma unroll
              for (int j = 0; j < 16; j++) {
                uint32_t& a = acc[LOG * p2 + h2][j];
                if constexpr (Q8)  // hi.hi + floor((hi.lo + lo.hi) / 256), still an integer
                  a = (uint32_t)((int)a + ((int)lo[h2][j] >> 8));
                else
                  a = __float_as_uint(__fadd_rn(__uint_as_float(a), __uint_as_float(lo[h2][j])));
              }
          }
          tc_fence_before();
          mbar_arrive(tempty);
        }
        if (!IP || PROD) {
#pragma unroll
          for (int u = 0; u < HALF / 32; u++) cns[u * 32 + lane] = cnv[u];
          __syncwarp();
        }
        // Top-k mode scores the groups its vote selects straight from TMEM
        // in a rolled loop (its group code is long: unrolled eight times it
        // no longer fits the instruction cache) and frees TMEM after the
        // tile; top-1 mode scores the drained registers in an unrolled loop.
        // The scoring of group g of this half tile, its 16 values in h.
        auto score_group = [&](const uint32_t(&h)[16], const int g) {
          if constexpr (PROD) {
            // The largest weighted product of the columns other than the own.
            const long cb = col0 + g * 16;
#pragma unroll
            for (int j = 0; j < 16; j++) {
              const float v = __uint_as_float(h[j]) * cns[g * 16 + j];
              if (cb + j != own_col && cb + j < P.k && v > pm) {
                pm = v;
                pc = (uint32_t)(cb + j);
              }
            }
            return;
          }
          float s[16];
          if constexpr (TOPK) {
            // Inner product: the accumulator is the screened value (fixed
            // point: an integer in units of 65536, converted here).
#pragma unroll
            for (int j = 0; j < 16; j++)
              s[j] = Q8 ? __int2float_rn((int)h[j]) : __uint_as_float(h[j]);
          } else {
            const float4* c4 = reinterpret_cast<const float4*>(cns + g * 16);
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              const float4 cv = IP ? make_float4(0.f, 0.f, 0.f, 0.f) : c4[j / 4];
              const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
              for (int w = 0; w < 4; w++) {
                // hi + lo, added in the drain (fixed point: an integer in units of
                // 65536, converted here once)
                const float v = Q8 ? __int2float_rn((int)h[j + w]) : __uint_as_float(h[j + w]);
                s[j + w] = __fmaf_rn(m2f, v, cc[w]);
              }
            }
          }
          const int lim = P.k - (col0 + g * 16);
          if (lim < 16) {  // warp-uniform: only the last, partial group of the centroids
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (j >= lim) s[j] = IP ? -INFINITY : INFINITY;
          }
          if (TOPK && P.exclude_self) {
            const long rel = gid - (P.col_gid0 + col0 + g * 16);  // the row's own column
            if ((unsigned long)rel < 16ul) {
#pragma unroll
              for (int j = 0; j < 16; j++)
                if (rel == j) s[j] = -INFINITY;
            }
          }
          // The group's best moves the threshold first.
          float t[8];
#pragma unroll
          for (int j = 0; j < 8; j++) t[j] = IP ? fmaxf(s[j], s[j + 8]) : fminf(s[j], s[j + 8]);
#pragma unroll
          for (int w2 = 4; w2 >= 1; w2 >>= 1)
#pragma unroll
            for (int j = 0; j < w2; j++) t[j] = IP ? fmaxf(t[j], t[j + w2]) : fminf(t[j], t[j + w2]);
          if constexpr (TOPK) {
            // Nothing in the group reaches any lane's window (thr <= kth): no
            // best-kk update and no admission, the usual case once the rows
            // have seen a few tiles.
            if (!__any_sync(0xFFFFFFFFu, collect && t[0] >= thr)) return;
            // Columns above the kk-th best enter the best-kk values. One such
            // column in the group (the usual case once the row has seen a few
            // tiles) is the group's best, t[0]; two or more are read back from
            // the warp's slab.
            const bool upd = collect && t[0] > kth;
            uint32_t m_up = 0;
            if (upd) {
#pragma unroll
              for (int j = 0; j < 16; j++) m_up |= (uint32_t)(s[j] > kth) << j;
            }
            const int nup = __popc(m_up);
            if (nup == 1) {
              kv_insert(kv, t[0]);
              kth = kv[0];
            }
            if (__any_sync(0xFFFFFFFFu, nup > 1)) {
#pragma unroll
              for (int j = 0; j < 16; j++) svs[j * 32] = s[j];
              __syncwarp();
              if (nup > 1) {
                while (m_up) {
                  const int j = __ffs(m_up) - 1;
                  m_up &= m_up - 1;
                  const float cv = svs[j * 32];
                  if (!(cv > kv[0])) continue;
                  kv_insert(kv, cv);
                  kth = kv[0];
                }
              }
              __syncwarp();
            }
            thr = kth > -INFINITY ? __fsub_rd(kth, off) : -INFINITY;
          } else if (IP ? (t[0] > best) : (t[0] < best)) {
            best = t[0];
            thr = IP ? __fsub_rd(best, off) : __fadd_ru(best, off);
          }
          uint32_t adm = 0;
#pragma unroll
          for (int j = 0; j < 16; j++)
            adm |= (uint32_t)(TOPK ? (s[j] >= thr && s[j] > -INFINITY)
                                   : (IP ? (s[j] >= thr) : (s[j] <= thr))) << j;
          if (!collect) adm = 0;
          // Appends. A single admitted column is the group's best, t[0], and
          // is appended directly; for two or more the warp stages the group's
          // values in its slab and each such lane walks its set bits, reading
          // the values back by index.
          const int na = __popc(adm);
          if (TOPK && na == 1) {
            if (cnt + 1 > LCAP) cnt = compact_list<IP>(row_list, P.m, cnt, thr);
            if (cnt < LCAP)
              row_list[cnt * P.m] =
                  make_uint2((uint32_t)(col0 + g * 16 + __ffs(adm) - 1), __float_as_uint(t[0]));
            overflow |= cnt >= LCAP;
            cnt += cnt < LCAP;
          }
          if (__any_sync(0xFFFFFFFFu, TOPK ? na > 1 : na > 0)) {
#pragma unroll
            for (int j = 0; j < 16; j++) svs[j * 32] = s[j];
            __syncwarp();
            if (TOPK ? na > 1 : na > 0) {
              if (cnt + (uint32_t)na > LCAP) cnt = compact_list<IP>(row_list, P.m, cnt, thr);
              const uint32_t base = (uint32_t)(col0 + g * 16);
              while (adm) {
                const int j = __ffs(adm) - 1;
                adm &= adm - 1;
                if (cnt < LCAP) row_list[cnt * P.m] = make_uint2(base + j, __float_as_uint(svs[j * 32]));
                overflow |= cnt >= LCAP;
                cnt += cnt < LCAP;
              }
            }
            __syncwarp();
          }
        };
        if constexpr (TOPK) {
          // Fixed-point top-k: the groups are voted on first, one at a time
          // straight from TMEM (each group's largest value hi + floor(lo /
          // 256), an integer maximum and one conversion, against the row's
          // threshold as the tile began; thresholds only rise, so a group no
          // lane votes for would be skipped by the full scoring as well).
          // Only the groups some lane wants are scored in full, each read
          // again from TMEM in a rolled loop, and TMEM is released after
          // them (the best-kk state leaves no room to hold the tile in
          // registers).
          uint32_t need = 0;
#pragma unroll
          for (int g = 0; g < HALF / 16; g++) {
            if (g < ngr) {
              uint32_t h[16], l[16];
              tmem_ld16(lane_base + (uint32_t)(g * 16), h);
              tmem_ld16(lane_base + (uint32_t)(BN + g * 16), l);
              tmem_wait();
              tmem_tie(h);
              tmem_tie(l);
              int mx = (int)h[0] + ((int)l[0] >> 8);
#pragma unroll
              for (int j = 1; j < 16; j++) mx = max(mx, (int)h[j] + ((int)l[j] >> 8));
              need |= (uint32_t)__any_sync(0xFFFFFFFFu, collect && __int2float_rn(mx) >= thr) << g;
            }
          }
#pragma unroll 1
          while (need) {
            const int g = __ffs(need) - 1;
            need &= need - 1;
            uint32_t h[16], l[16];
            tmem_ld16(lane_base + (uint32_t)(g * 16), h);
            tmem_ld16(lane_base + (uint32_t)(BN + g * 16), l);
            tmem_wait();
            tmem_tie(h);
            tmem_tie(l);
#pragma unroll
            for (int j = 0; j < 16; j++) h[j] = (uint32_t)((int)h[j] + ((int)l[j] >> 8));
            score_group(h, g);
          }
          tc_fence_before();
          mbar_arrive(tempty);
        } else {
#pragma unroll
          for (int g = 0; g < HALF / 16; g++) {
            if (g >= ngr) break;
            score_group(acc[g], g);
          }
        }
      }
      if (PROD) {
        if (live) {
          P.pmax[L * P.m + i] = collect && !stop ? pm : NAN;
          P.pcol[L * P.m + i] = pc;
        }
      } else if (live) {
        // A half tile past the last centroid (k <= HALF, or a last part
        // whose one tile has HALF centroids or fewer) holds no centroid at
        // all: its list is empty and its threshold the identity, not a
        // fallback.
        const bool no_columns = nt0 * BN + hf * HALF >= P.k;
        const bool ok = collect && !stop && !overflow && !*abort_flag &&
                        (TOPK || isfinite(best) || no_columns);
        if (ok) P.cand_thr[L * P.m + i] = thr;
        P.cand_cnt[L * P.m + i] = ok ? cnt : FALLBACK;
        if constexpr (TOPK) {
          float* kvo = P.kvals + (L * P.m + i) * KMAX;
#pragma unroll
          for (int a = 0; a < KMAX; a++) kvo[a] = kv[a];
          if (hf == 0) P.roff[i] = off;
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(P.status, ST_WAIT_TIMEOUT);
}

// ---------------------------------------------------------------- exact stage

// Warp-aggregated append: every lane of a full warp calls this with its own
// count n (possibly 0); one atomic per warp reserves the slots, and each lane
// gets the first of its own.
__device__ __forceinline__ uint32_t warp_append(uint32_t* counter, uint32_t n) {
  const int lane = threadIdx.x & 31;
  uint32_t incl = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  uint32_t base = 0;
  if (lane == 31 && incl) base = atomicAdd(counter, incl);
  return __shfl_sync(0xFFFFFFFFu, base, 31) + incl - n;
}

// Key of (v, j): larger key = better for IP (max v, then min j); smaller key
// = better for L2 (min v, then min j). -0.0 counts as +0.0: they compare
// equal in the CPU's scan, so the lower id must decide.
template <bool IP>
__device__ __forceinline__ unsigned long long result_key(float v, uint32_t j) {
  if (v == 0.0f) v = 0.0f;
  const uint32_t u = __float_as_uint(v);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (IP ? (uint32_t)~j : j);
}

// The key of the CPU scan's starting point (-inf / +inf with id 0): only a
// strictly better value replaces it, exactly as in the sequential scan.
template <bool IP>
__device__ __forceinline__ unsigned long long scan_start_key() {
  return result_key<IP>(IP ? -INFINITY : INFINITY, 0u);
}

// Each row's candidates (from its nl lists, two per part: one per part and
// half tile) still inside its final window become (row, centroid) pairs; the
// window is the tightest of the lists' thresholds, the one of the row's
// overall best. Rows with none, with more than SURV, or marked for the
// fallback go to the exact list, whose key starts at the scan's starting
// point. The row's pair key starts at the identity of its reduction. Launched
// with 256 threads a block at no more than 40 registers a thread, so that
// six blocks share an SM and a whole C2 pass's rows are in flight at once (at
// 107 registers, two blocks an SM made it three waves of dependent loads);
// the entries are read twice, to count and to write, the second time from
// L2. The pair slots are reserved with one atomic per block (the per-warp
// atomics on one counter serialised).
constexpr int MAX_PARTS = 4;
template <bool IP>
__global__ void __launch_bounds__(256, 6) k_collect(
    long p0, long m, uint32_t k, int nl, const uint2* __restrict__ cand,
    const uint32_t* __restrict__ cand_cnt, const float* __restrict__ cand_thr,
    uint2* __restrict__ pairs, uint32_t* __restrict__ pair_count,
    unsigned long long* __restrict__ rkey, uint32_t* __restrict__ list,
    uint32_t* __restrict__ list_count, unsigned long long* __restrict__ lkey,
    uint32_t* __restrict__ bad, unsigned long long* __restrict__ counters,
    uint32_t* __restrict__ status) {
  pdl_wait();
  __shared__ uint32_t wsum[8], wbase[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < m;
  // The lists' counts and thresholds, all loads in flight together (a
  // fallback list's threshold is not written and not used).
  bool fb = !live;
  float thr = IP ? -INFINITY : INFINITY;
  if (live) {
    for (int h = 0; h < nl; h++) {
      const uint32_t c = __ldg(cand_cnt + h * m + i);
      const float th = __ldg(cand_thr + h * m + i);
      if (c == FALLBACK) {
        fb = true;
      } else if (c > CAP) {
        atomicOr(status, ST_BAD_STATE);
        fb = true;
      }
      thr = IP ? fmaxf(thr, th) : fminf(thr, th);
    }
  }
  // Count the entries inside the window, four loads at a time.
  uint32_t ns = 0;
  bool bad_entry = false;
  if (!fb) {
    for (int h = 0; h < nl; h++) {
      const uint32_t c = __ldg(cand_cnt + h * m + i);
      const uint2* lst = cand + (long)h * CAP * m + i;
      for (uint32_t e0 = 0; e0 < c; e0 += 4) {
        uint2 en[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
          en[u] = e0 + u < c ? __ldg(lst + (e0 + u) * m) : make_uint2(0u, __float_as_uint(NAN));
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const float sv = __uint_as_float(en[u].y);
          bad_entry |= en[u].x >= k;
          ns += IP ? (sv >= thr) : (sv <= thr);
        }
      }
    }
  }
  if (bad_entry) atomicOr(status, ST_BAD_STATE);
  fb = fb || bad_entry || ns == 0 || ns > SURV;
  const bool listed = live && fb;
  const uint32_t np = live && !fb ? ns : 0;
  if (live) {
    rkey[i] = IP ? 0ull : ~0ull;
    bad[i] = 0u;
  }
  const uint32_t lp = warp_append(list_count, listed ? 1u : 0u);
  if (listed) {
    list[lp] = (uint32_t)(p0 + i);
    lkey[lp] = scan_start_key<IP>();
  }
  // Pair slots: this lane's offset in its warp, the warp's in the block, and
  // the block's from one atomic.
  uint32_t incl = np;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    const int nw = (int)(blockDim.x >> 5);
    for (int w2 = 0; w2 < nw; w2++) {
      const uint32_t v = wsum[w2];
      wbase[w2] = run;
      run += v;
    }
    const uint32_t base = run ? atomicAdd(pair_count, run) : 0u;
    for (int w2 = 0; w2 < nw; w2++) wbase[w2] += base;
    if (run) atomicAdd(&counters[2], (unsigned long long)run);
  }
  __syncthreads();
  uint32_t w = wbase[warp] + incl - np;
  if (np) {
#pragma unroll 1
    for (int h = 0; h < nl; h++) {
      const uint32_t c = __ldg(cand_cnt + h * m + i);
      const uint2* lst = cand + (long)h * CAP * m + i;
#pragma unroll 4
      for (uint32_t e = 0; e < c; e++) {
        const uint2 en = __ldg(lst + e * m);
        const float sv = __uint_as_float(en.y);
        if (IP ? (sv >= thr) : (sv <= thr)) pairs[w++] = make_uint2((uint32_t)i, en.x);
      }
    }
  }
  const uint32_t nlisted = __reduce_add_sync(0xFFFFFFFFu, listed ? 1u : 0u);
  if (lane == 0 && nlisted) atomicAdd(&counters[1], (unsigned long long)nlisted);
}

// Exact FMA chain of row x against centroid c over d columns, loads kept
// several steps ahead of the dependent FMAs.
__device__ __forceinline__ float chain(const float* __restrict__ x, const float* __restrict__ c,
                                       int d) {
  float acc = 0.0f;
  if ((d & 3) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* c4 = reinterpret_cast<const float4*>(c);
    const int q = d / 4;
    int t = 0;
    for (; t + 4 <= q; t += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        a[u] = __ldg(x4 + t + u);
        b[u] = __ldg(c4 + t + u);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        acc = __fmaf_rn(a[u].x, b[u].x, acc);
        acc = __fmaf_rn(a[u].y, b[u].y, acc);
        acc = __fmaf_rn(a[u].z, b[u].z, acc);
        acc = __fmaf_rn(a[u].w, b[u].w, acc);
      }
    }
    for (; t < q; t++) {
      const float4 a = __ldg(x4 + t), b = __ldg(c4 + t);
      acc = __fmaf_rn(a.x, b.x, acc);
      acc = __fmaf_rn(a.y, b.y, acc);
      acc = __fmaf_rn(a.z, b.z, acc);
      acc = __fmaf_rn(a.w, b.w, acc);
    }
  } else {
    for (int t = 0; t < d; t++) acc = __fmaf_rn(__ldg(x + t), __ldg(c + t), acc);
  }
  return acc;
}

// Exact chains over the (row, centroid) pairs, one thread per pair. Each warp
// runs its own pipeline over its 32 pairs, with no barrier across warps: x
// and the centroid stream through the warp's shared memory in 32-column
// slices (cp.async, EX_STAGES slices in flight; each copy instruction moves
// four whole 128-byte row segments), and each 16-byte chunk q of pair slot r
// is stored at q ^ (r & 7) so that the per-lane LDS.128 reads are free of
// bank conflicts. Each pair folds (value, id) into its row's key with an
// atomic max / min.
// 8 warps x 3 stages per SM (measured: a 2 warps x 12 stages shape was more
// than twice as slow on a training batch's pairs).
constexpr int EX_COLS = 32;
template <int WARPS, int STAGES>
constexpr size_t ex_smem() {
  return (size_t)WARPS * STAGES * 2 * 32 * EX_COLS * sizeof(float);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool IP, int EX_WARPS = 8, int EX_STAGES = 3>
__global__ void __launch_bounds__(EX_WARPS * 32) k_pairs(
    const float* __restrict__ x, int d, const uint32_t* __restrict__ ids, long p0,
    const float* __restrict__ c, const float* __restrict__ cn, const float* __restrict__ xnorm_row,
    const uint2* __restrict__ pairs, const uint32_t* __restrict__ pair_count, long m, uint32_t k,
    unsigned long long* __restrict__ rkey, float* __restrict__ xn_pos,
    uint32_t* __restrict__ bad, uint32_t* __restrict__ status, float* __restrict__ pval) {
  pdl_wait();
  extern __shared__ __align__(16) float ex_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int EX_WARP_FLOATS = EX_STAGES * 2 * 32 * EX_COLS;  // x and c slices of one warp
  float* xs = ex_smem + warp * EX_WARP_FLOATS;  // [stage][pair][32]
  float* cs = xs + EX_STAGES * 32 * EX_COLS;     // [stage][pair][32]
  const long np = (long)*pair_count;
  const int nsl = d / EX_COLS;
  const bool want_xn = !IP && !xnorm_row;
  const long stride = (long)gridDim.x * EX_WARPS;
  // Consecutive 32-pair tiles go to different SMs, so that a small pass
  // (a training batch) spreads over all of them. (Measured: an L2 prefetch of
  // each tile's whole rows made large passes slower.)
  for (long wt = (long)warp * gridDim.x + blockIdx.x; wt * 32 < np; wt += stride) {
    const long pi = wt * 32 + lane;
    bool mine = pi < np;
    uint2 pr = make_uint2(0, 0);
    long row = 0;
    if (mine) {
      pr = pairs[pi];
      if (pr.x >= m || pr.y >= k) {
        atomicOr(status, ST_BAD_STATE);
        pr = make_uint2(0, 0);
        mine = false;
      }
      row = ids ? (long)ids[p0 + pr.x] : p0 + pr.x;
    }
    // Slots past the pair count read row 0 / centroid 0 harmlessly and write
    // nothing. This lane copies 16-byte chunk q = lane % 8 of pair slots
    // r = 4 u + lane / 8 (u = 0 .. 7) of every x and c slice; the slots' row
    // addresses come from their lanes by shuffle, once per tile, and stay in
    // registers with the chunks' shared-memory offsets.
    const unsigned long long xrow = (unsigned long long)(x + row * (long)d);
    const unsigned long long crow = (unsigned long long)(c + (long)pr.y * d);
    const int q = lane & 7;
    const float* xsrc[8];
    const float* csrc[8];
    int soff[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int r = u * 4 + (lane >> 3);
      xsrc[u] = reinterpret_cast<const float*>(__shfl_sync(0xFFFFFFFFu, xrow, r)) + q * 4;
      csrc[u] = reinterpret_cast<const float*>(__shfl_sync(0xFFFFFFFFu, crow, r)) + q * 4;
      soff[u] = r * EX_COLS + ((q ^ (r & 7)) << 2);
    }
    auto issue = [&](int sl) {
      if (sl < nsl) {
        const int sbase = (sl % EX_STAGES) * 32 * EX_COLS;
        const int g = sl * EX_COLS;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          cp_async16(xs + sbase + soff[u], xsrc[u] + g);
          cp_async16(cs + sbase + soff[u], csrc[u] + g);
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < EX_STAGES - 1; s++) issue(s);
    float acc = 0.0f, xn = -0.0f;
    for (int sl = 0; sl < nsl; sl++) {
      issue(sl + EX_STAGES - 1);
      cp_async_wait<EX_STAGES - 1>();
      __syncwarp();
      const int base = (sl % EX_STAGES * 32 + lane) * EX_COLS;
      const float4* xr4 = reinterpret_cast<const float4*>(xs + base);
      const float4* cr4 = reinterpret_cast<const float4*>(cs + base);
      // All sixteen loads first, so that their latencies overlap.
      float4 av[8], bv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const int pq = q ^ (lane & 7);
        av[q] = xr4[pq];
        bv[q] = cr4[pq];
      }
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const float4 a = av[q], b = bv[q];
        acc = __fmaf_rn(a.x, b.x, acc);
        acc = __fmaf_rn(a.y, b.y, acc);
        acc = __fmaf_rn(a.z, b.z, acc);
        acc = __fmaf_rn(a.w, b.w, acc);
        if (want_xn) {
          // The row's sum of squares in the CPU order (sequential, no FMA).
          xn = __fadd_rn(xn, __fmul_rn(a.x, a.x));
          xn = __fadd_rn(xn, __fmul_rn(a.y, a.y));
          xn = __fadd_rn(xn, __fmul_rn(a.z, a.z));
          xn = __fadd_rn(xn, __fmul_rn(a.w, a.w));
        }
      }
      __syncwarp();  // the slot is refilled next iteration
    }
    cp_async_wait<0>();
    if (mine && pval) {
      pval[pi] = acc;  // top-k mode: every pair's exact inner product
    } else if (mine) {
      const float v = IP ? acc : __fsub_rn(__ldg(cn + pr.y), __fmul_rn(2.0f, acc));
      if (!isfinite(v)) {
        bad[pr.x] = 1;  // an overflowing chain: the exact list reproduces the CPU here
      } else if (IP) {
        atomicMax(rkey + pr.x, result_key<IP>(v, pr.y));
      } else {
        atomicMin(rkey + pr.x, result_key<IP>(v, pr.y));
      }
      if (want_xn) xn_pos[pr.x] = xn;  // the same value from every pair of the row
    }
    __syncwarp();  // the next tile refills the slices
  }
}

// The same for d % 32 != 0: one thread per pair reads its operands directly.
template <bool IP>
__global__ void k_pairs_plain(const float* __restrict__ x, int d, const uint32_t* __restrict__ ids,
                              long p0, const float* __restrict__ c, const float* __restrict__ cn,
                              const float* __restrict__ xnorm_row, const uint2* __restrict__ pairs,
                              const uint32_t* __restrict__ pair_count, long m, uint32_t k,
                              unsigned long long* __restrict__ rkey, float* __restrict__ xn_pos,
                              uint32_t* __restrict__ bad, uint32_t* __restrict__ status,
                              float* __restrict__ pval) {
  pdl_wait();
  const long np = (long)*pair_count;
  for (long pi = (long)blockIdx.x * blockDim.x + threadIdx.x; pi < np;
       pi += (long)gridDim.x * blockDim.x) {
    const uint2 pr = pairs[pi];
    if (pr.x >= m || pr.y >= k) {
      atomicOr(status, ST_BAD_STATE);
      continue;
    }
    const long row = ids ? (long)ids[p0 + pr.x] : p0 + pr.x;
    const float* xr = x + row * (long)d;
    const float acc = chain(xr, c + (long)pr.y * d, d);
    if (pval) {
      pval[pi] = acc;  // top-k mode
      continue;
    }
    const float v = IP ? acc : __fsub_rn(__ldg(cn + pr.y), __fmul_rn(2.0f, acc));
    if (!isfinite(v)) {
      bad[pr.x] = 1;
    } else if (IP) {
      atomicMax(rkey + pr.x, result_key<IP>(v, pr.y));
    } else {
      atomicMin(rkey + pr.x, result_key<IP>(v, pr.y));
    }
    if (!IP && !xnorm_row) {
      float xn = -0.0f;
      for (int u = 0; u < d; u++) {
        const float a = __ldg(xr + u);
        xn = __fadd_rn(xn, __fmul_rn(a, a));
      }
      xn_pos[pr.x] = xn;
    }
  }
}

// Decode a result key back to (value, id).
template <bool IP>
__device__ __forceinline__ float key_value(unsigned long long key, uint32_t& j) {
  const uint32_t ord = (uint32_t)(key >> 32);
  const uint32_t u = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
  j = IP ? ~(uint32_t)key : (uint32_t)key;
  return __uint_as_float(u);
}

// Labels and scores from the rows' keys; rows whose chains overflowed join
// the exact list. Launched with whole warps.
template <bool IP>
__global__ void __launch_bounds__(256) k_finish(
    const uint32_t* __restrict__ ids, long p0, long m, const float* __restrict__ xnorm_row,
    const float* __restrict__ xn_pos, const unsigned long long* __restrict__ rkey,
    const uint32_t* __restrict__ bad, uint32_t* __restrict__ labels, float* __restrict__ scores,
    uint32_t* __restrict__ list, uint32_t* __restrict__ list_count,
    unsigned long long* __restrict__ lkey, unsigned long long* __restrict__ counters) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < m;
  const bool listed = live && bad[i];
  const uint32_t lp = warp_append(list_count, listed ? 1u : 0u);
  const uint32_t nl = __reduce_add_sync(0xFFFFFFFFu, listed ? 1u : 0u);
  if ((threadIdx.x & 31) == 0 && nl) atomicAdd(&counters[1], (unsigned long long)nl);
  if (listed) {
    list[lp] = (uint32_t)(p0 + i);
    lkey[lp] = scan_start_key<IP>();
    return;
  }
  if (!live) return;
  const unsigned long long key = rkey[i];
  if (key == (IP ? 0ull : ~0ull)) return;  // on the list already
  uint32_t j;
  const float v = key_value<IP>(key, j);
  float score = v;
  if (!IP) {
    const long row = ids ? (long)ids[p0 + i] : p0 + i;
    score = fmaxf(__fadd_rn(xnorm_row ? xnorm_row[row] : xn_pos[i], v), 0.0f);
  }
  labels[p0 + i] = j;
  scores[p0 + i] = score;
}

// The exact list: rows the screen could not certify, scanned against every
// centroid. Work items are (listed row, block of LS_C centroids), one thread
// per centroid: the row's 32-column slice and the centroids' slices stream
// through shared memory (cp.async, LS_STAGES slices in flight; the same XOR
// layout as the pair kernel), each thread runs its centroid's FMA chain over
// all d columns, and the block folds its best (value, id) into the row's key.
// Keys start at the scan's starting point and skip NaN values, so the atomic
// reduction reproduces the sequential strict scan with its lower-id rule.
constexpr int LS_C = 128, LS_STAGES = 4;
constexpr size_t LS_SMEM = (size_t)LS_STAGES * (LS_C + 1) * EX_COLS * sizeof(float);

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}

template <bool IP>
__global__ void __launch_bounds__(LS_C) k_list(
    const float* __restrict__ x, long n, int d, const uint32_t* __restrict__ ids,
    const float* __restrict__ c, const float* __restrict__ cn, long k,
    const uint32_t* __restrict__ list, const uint32_t* __restrict__ list_count,
    unsigned long long* __restrict__ lkey, const float* __restrict__ xnorm_row,
    float* __restrict__ lxn, uint32_t* __restrict__ status) {
  pdl_wait();
  extern __shared__ __align__(16) float ls_smem[];
  float* cs = ls_smem;                                 // [stage][LS_C][32]
  float* xs = ls_smem + LS_STAGES * LS_C * EX_COLS;    // [stage][32]
  __shared__ unsigned long long red[LS_C / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long kch = (k + LS_C - 1) / LS_C;
  const long total = (long)*list_count * kch;
  const int nsl = (d + EX_COLS - 1) / EX_COLS;
  const bool v16 = (d & 3) == 0;  // rows start on 16-byte boundaries
  for (long w = blockIdx.x; w < total; w += gridDim.x) {
    const long ent = w / kch;
    const long j0 = (w - ent * kch) * LS_C;
    // The first centroid block's thread 0 also sums the row's squares in the
    // CPU order (sequential, no FMA) when the caller has no row norms.
    const bool sum_xn = !IP && !xnorm_row && j0 == 0 && t == 0;
    long row = list[ent];
    if (ids) row = ids[row];
    if (row >= n) {
      atomicOr(status, ST_BAD_ROW);
      row = 0;
    }
    const float* xr = x + row * (long)d;
    auto issue = [&](int sl) {
      if (sl < nsl) {
        const int st = sl % LS_STAGES;
        const int g0 = sl * EX_COLS;
        float* cst = cs + st * LS_C * EX_COLS;
        if (v16) {
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const int idx = u * LS_C + t;  // 0 .. 1023
            const int r = idx >> 3, q = idx & 7;
            const int g = g0 + q * 4;
            if (j0 + r < k && g < d)
              cp_async16(cst + r * EX_COLS + (q ^ (r & 7)) * 4, c + (j0 + r) * (long)d + g);
          }
          if (t < 8 && g0 + t * 4 < d) cp_async16(xs + st * EX_COLS + t * 4, xr + g0 + t * 4);
        } else {
#pragma unroll 4
          for (int u = 0; u < 32; u++) {
            const int idx = u * LS_C + t;  // 0 .. 4095
            const int r = idx >> 5, cc = idx & 31;
            const int g = g0 + cc;
            if (j0 + r < k && g < d)
              cp_async4(cst + r * EX_COLS + (((cc >> 2) ^ (r & 7)) << 2) + (cc & 3),
                        c + (j0 + r) * (long)d + g);
          }
          if (t < 32 && g0 + t < d) cp_async4(xs + st * EX_COLS + t, xr + g0 + t);
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < LS_STAGES - 1; s++) issue(s);
    float acc = 0.0f, xn = -0.0f;
    for (int sl = 0; sl < nsl; sl++) {
      issue(sl + LS_STAGES - 1);
      cp_async_wait<LS_STAGES - 1>();
      __syncthreads();
      const int st = sl % LS_STAGES;
      const float* crow = cs + (st * LS_C + t) * EX_COLS;
      const float* xsl = xs + st * EX_COLS;
      const int kmax = min(EX_COLS, d - sl * EX_COLS);
      if (sum_xn)
        for (int cc = 0; cc < kmax; cc++) xn = __fadd_rn(xn, __fmul_rn(xsl[cc], xsl[cc]));
      if (kmax == EX_COLS) {
        const float4* x4 = reinterpret_cast<const float4*>(xsl);
        const float4* c4 = reinterpret_cast<const float4*>(crow);
#pragma unroll
        for (int q = 0; q < 8; q++) {
          const float4 a = x4[q], b = c4[q ^ (t & 7)];
          acc = __fmaf_rn(a.x, b.x, acc);
          acc = __fmaf_rn(a.y, b.y, acc);
          acc = __fmaf_rn(a.z, b.z, acc);
          acc = __fmaf_rn(a.w, b.w, acc);
        }
      } else {
        for (int cc = 0; cc < kmax; cc++)
          acc = __fmaf_rn(xsl[cc], crow[(((cc >> 2) ^ (t & 7)) << 2) + (cc & 3)], acc);
      }
      __syncthreads();  // the slot is refilled next iteration
    }
    cp_async_wait<0>();
    if (sum_xn) lxn[ent] = xn;
    const long j = j0 + t;
    unsigned long long key = scan_start_key<IP>();
    if (j < k) {
      const float v = IP ? acc : __fsub_rn(__ldg(cn + j), __fmul_rn(2.0f, acc));
      if (!isnan(v)) key = result_key<IP>(v, (uint32_t)j);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, key, o);
      key = IP ? max(key, other) : min(key, other);
    }
    if (lane == 0) red[warp] = key;
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int u = 1; u < LS_C / 32; u++) key = IP ? max(key, red[u]) : min(key, red[u]);
      if (key != scan_start_key<IP>()) {
        if (IP)
          atomicMax(lkey + ent, key);
        else
          atomicMin(lkey + ent, key);
      }
    }
  }
}

// Labels and scores of the listed rows from their keys.
template <bool IP>
__global__ void k_list_finish(const float* __restrict__ x, long n, int d,
                              const uint32_t* __restrict__ ids,
                              const uint32_t* __restrict__ list,
                              const uint32_t* __restrict__ list_count,
                              const unsigned long long* __restrict__ lkey,
                              const float* __restrict__ xnorm_row, const float* __restrict__ lxn,
                              uint32_t* __restrict__ labels, float* __restrict__ scores) {
  pdl_wait();
  const long cnt = (long)*list_count;
  for (long ent = (long)blockIdx.x * blockDim.x + threadIdx.x; ent < cnt;
       ent += (long)gridDim.x * blockDim.x) {
    const long p = list[ent];
    uint32_t j;
    const float v = key_value<IP>(lkey[ent], j);
    float score = v;
    if (!IP) {
      long row = ids ? (long)ids[p] : p;
      if (row >= n) row = 0;  // reported by the scan kernel
      const float xn = xnorm_row ? xnorm_row[row] : lxn[ent];
      score = fmaxf(__fadd_rn(xn, v), 0.0f);
    }
    labels[p] = j;
    scores[p] = score;
  }
}

// ---------------------------------------------------------------- top-k stage

// Top-k mode: a row's window is 2e below the kk-th best of the union of its
// two halves' best-kk values (the row's screened kk-th best). Its listed
// columns still inside become (row, column) pairs, contiguous per row
// (pstart, pcnt); rows with none, more than SURV, or marked for the fallback
// go to the full scan (pcnt 0). Launched with whole warps.
__global__ void __launch_bounds__(256) k_collect_topk(
    long p0, long m, uint32_t n, int kk, const uint2* __restrict__ cand,
    const uint32_t* __restrict__ cand_cnt, const float* __restrict__ kvals,
    const float* __restrict__ roff, uint2* __restrict__ pairs, uint32_t* __restrict__ pair_count,
    uint32_t* __restrict__ pstart, uint32_t* __restrict__ pcnt, uint32_t* __restrict__ list,
    uint32_t* __restrict__ list_count, unsigned long long* __restrict__ counters,
    uint32_t* __restrict__ status) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < m;
  uint32_t cnt[2] = {0, 0};
  bool fb = !live;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    cnt[h] = live ? cand_cnt[h * m + i] : 0;
    if (cnt[h] == FALLBACK) {
      fb = true;
      cnt[h] = 0;
    } else if (cnt[h] > CAP_TOPK) {
      atomicOr(status, ST_BAD_STATE);
      fb = true;
      cnt[h] = 0;
    }
  }
  float thr = -INFINITY;
  uint32_t ns = 0;
  if (!fb) {
    // The kk-th largest of the two halves' best-kk values (each ascending in
    // slots 0 .. kk - 1): a merge from the top.
    const float* a = kvals + i * KMAX;
    const float* b = kvals + (m + i) * KMAX;
    int ia = kk - 1, ib = kk - 1;
    float kth = -INFINITY;
    for (int t = 0; t < kk; t++) {
      const float va = ia >= 0 ? a[ia] : -INFINITY;
      const float vb = ib >= 0 ? b[ib] : -INFINITY;
      if (va >= vb) {
        kth = va;
        ia--;
      } else {
        kth = vb;
        ib--;
      }
    }
    thr = kth > -INFINITY ? __fsub_rd(kth, roff[i]) : -INFINITY;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint2* lst = cand + (long)h * CAP_TOPK * m + i;
      for (uint32_t e = 0; e < cnt[h]; e++) {
        const uint2 en = lst[e * m];
        const float sv = __uint_as_float(en.y);
        if (en.x >= n) fb = true;
        ns += sv >= thr && sv > -INFINITY;
      }
    }
    if (fb) atomicOr(status, ST_BAD_STATE);
  }
  fb = fb || ns == 0 || ns > SURV;
  const bool listed = live && fb;
  const uint32_t np = live && !fb ? ns : 0;
  const uint32_t lp = warp_append(list_count, listed ? 1u : 0u);
  if (listed) list[lp] = (uint32_t)(p0 + i);
  uint32_t w = warp_append(pair_count, np);
  if (live) {
    pstart[i] = w;
    pcnt[i] = np;
  }
  if (np) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint2* lst = cand + (long)h * CAP_TOPK * m + i;
      for (uint32_t e = 0; e < cnt[h]; e++) {
        const uint2 en = lst[e * m];
        const float sv = __uint_as_float(en.y);
        if (sv >= thr && sv > -INFINITY) pairs[w++] = make_uint2((uint32_t)i, en.x);
      }
    }
  }
  const uint32_t nl = __reduce_add_sync(0xFFFFFFFFu, listed ? 1u : 0u);
  const uint32_t nps = __reduce_add_sync(0xFFFFFFFFu, np);
  if ((threadIdx.x & 31) == 0) {
    if (nl) atomicAdd(&counters[1], (unsigned long long)nl);
    if (nps) atomicAdd(&counters[2], (unsigned long long)nps);
  }
}

// Each row's best kk of its pairs' exact inner products by (larger score,
// then lower id); NaN and -inf never enter, missing entries stay
// (0xFFFFFFFF, -inf). Rows of the full scan (pcnt 0) are written there.
__global__ void k_topk_finish(long p0, long m, int kk, uint32_t id0,
                              const uint32_t* __restrict__ pstart,
                              const uint32_t* __restrict__ pcnt, const uint2* __restrict__ pairs,
                              const float* __restrict__ pval, uint32_t* __restrict__ ids,
                              float* __restrict__ sims) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const uint32_t np = pcnt[i];
  if (np == 0) return;
  float ls[KMAX];
  uint32_t li[KMAX];
#pragma unroll
  for (int a = 0; a < KMAX; a++) {
    ls[a] = -INFINITY;
    li[a] = 0xFFFFFFFFu;
  }
  const uint32_t s0 = pstart[i];
  for (uint32_t t = 0; t < np; t++) {
    float cv = pval[s0 + t];
    uint32_t cj = pairs[s0 + t].y;
    if (!(cv > -INFINITY)) continue;
#pragma unroll
    for (int a = 0; a < KMAX; a++) {
      const bool b = a < kk && (cv > ls[a] || (cv == ls[a] && cj < li[a]));
      const float tv = ls[a];
      const uint32_t tj = li[a];
      ls[a] = b ? cv : tv;
      li[a] = b ? cj : tj;
      cv = b ? tv : cv;
      cj = b ? tj : cj;
    }
  }
  const long o = (p0 + i) * (long)kk;
#pragma unroll
  for (int a = 0; a < KMAX; a++) {
    if (a < kk) {
      ids[o + a] = li[a] == 0xFFFFFFFFu ? li[a] : li[a] + id0;  // global ids
      sims[o + a] = li[a] == 0xFFFFFFFFu ? -INFINITY : ls[a];
    }
  }
}

// Gather the rows of listed queries (global positions) into a dense block.
__global__ void k_gather_queries(const float* __restrict__ q, int d, const uint32_t* __restrict__ list,
                                 long L, float* __restrict__ out) {
  pdl_wait();
  const long t = (long)blockIdx.y * gridDim.x + blockIdx.x;
  if (t >= L) return;
  const float* src = q + (long)list[t] * d;
  float* dst = out + t * d;
  for (int c = threadIdx.x; c < d; c += blockDim.x) dst[c] = src[c];
}

// Scatter the full scan's results of the listed queries into place.
__global__ void k_scatter_topk(const uint32_t* __restrict__ list, long L, int kk,
                               const uint32_t* __restrict__ tids, const float* __restrict__ tsims,
                               uint32_t* __restrict__ ids, float* __restrict__ sims) {
  pdl_wait();
  const long u = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= L * kk) return;
  const long t = u / kk, a = u - t * kk;
  const long o = (long)list[t] * kk + a;
  ids[o] = tids[u];
  sims[o] = tsims[u];
}

// ---------------------------------------------------------------- product stage

// Product mode: each row's column of the largest weighted product over the
// columns other than its own (over its lists; the lower column on ties), or
// 0xFFFFFFFF when there is none. Rows or centroids with non-finite values, or
// a screen that gave up: 0xFFFFFFFE.
__global__ void k_prod_finish(long p0, long m, int nl, const int* __restrict__ xexp,
                              const unsigned long long* __restrict__ cinfo, uint32_t cgen,
                              const float* __restrict__ pmax, const uint32_t* __restrict__ pcol,
                              uint32_t* __restrict__ best_out) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  uint32_t bc = 0xFFFFFFFEu;
  if (xexp[i] != XEXP_BAD && cinfo_word(cinfo, 2, cgen) == 0) {
    float vm = -INFINITY;
    bc = 0xFFFFFFFFu;
    for (int h = 0; h < nl; h++) {
      const float v = pmax[(long)h * m + i];
      const uint32_t c = pcol[(long)h * m + i];
      if (isnan(v)) {
        bc = 0xFFFFFFFEu;
        break;
      }
      if (c != 0xFFFFFFFFu && (v > vm || (v == vm && c < bc))) {
        vm = v;
        bc = c;
      }
    }
  }
  best_out[p0 + i] = bc;
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    EB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p)
      throw Error(EB_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// A 2-D FP16 tensor map over rows x dp (row stride dp*2 bytes) with a box of
// `box_rows` x 32 columns (64 bytes, 64-byte swizzle). The inner coordinate of
// every load is a multiple of 32 elements (64 bytes).
CUtensorMap make_map(const void* base, size_t rows, size_t dp, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)dp, (cuuint64_t)std::max<size_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)dp * 2};
  cuuint32_t box[2] = {(cuuint32_t)BKH, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(EB_ERROR, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

// The same for a fixed-point copy: int8 digits, dp8 bytes a row, boxes of
// 64 columns (64 bytes) by box_rows.
CUtensorMap make_map_q8(const void* base, size_t rows, size_t dp8, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)dp8, (cuuint64_t)std::max<size_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)dp8};
  cuuint32_t box[2] = {(cuuint32_t)BK8, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(EB_ERROR, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

// Dynamic shared memory limits are per-device, per-kernel attributes.
template <bool IP, bool TOPK, bool PROD = false, bool Q8 = false>
void set_smem(int device) {
  static uint64_t done = 0;  // one instance per kernel: the template parameters
  if (!(done >> device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_screen<IP, TOPK, PROD, Q8>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    done |= 1ull << device;
  }
}

template <bool IP, int WARPS, int STAGES>
void set_pairs_smem(int device) {
  static uint64_t done = 0;  // one instance per kernel shape
  if (!(done >> device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_pairs<IP, WARPS, STAGES>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)ex_smem<WARPS, STAGES>()));
    done |= 1ull << device;
  }
}

// The exact chains of the pairs of a pass of m rows (d % 32 == 0).
template <bool IP>
void launch_pairs(eb_engine* e, long m, const float* x, int d, const uint32_t* ids, long p0,
                  const float* c, const float* cn, const float* xnorm, const uint2* pairs,
                  const uint32_t* pair_count, uint32_t k, unsigned long long* rkey,
                  float* xn_pos, uint32_t* bad, float* pval) {
  const unsigned grid = (unsigned)e->num_sms;
  // Measured against 4-12 warps x 2-6 stages; on a training batch (about 18,000
  // pairs) 4 x 6 took 19.3 us against 16.7.
  constexpr int W = 8, S = 3;
  set_pairs_smem<IP, W, S>(e->device);
  launch_pdl(e, k_pairs<IP, W, S>, grid, W * 32, ex_smem<W, S>(), x, d, ids, p0, c, cn, xnorm, pairs, pair_count, m, k, rkey, xn_pos, bad, e->d_status, pval);
}

template <bool IP>
void set_list_smem(int device) {
  static uint64_t done = 0;
  if (!(done >> device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_list<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)LS_SMEM));
    done |= 1ull << device;
  }
}

template <bool IP, bool TOPK = false, bool PROD = false, bool Q8 = false>
void launch_screen(eb_engine* e, unsigned grid, const CUtensorMap& ah, const CUtensorMap& al,
                   const CUtensorMap& bh, const CUtensorMap& bl, const ScreenParams& P) {
  set_smem<IP, TOPK, PROD, Q8>(e->device);
  launch_pdl(e, k_screen<IP, TOPK, PROD, Q8>, grid, NTHREADS, SMEM_BYTES, ah, al, bh, bl, P);
}

// Scratch of the exact stage of one pass of m rows.
struct ExactScratch {
  int nl;  // candidate lists per row (2 per part)
  const uint2* cand;
  const uint32_t* cand_cnt;
  const float* cand_thr;
  uint2* pairs;
  uint32_t* pair_count;
  unsigned long long* rkey;
  uint32_t* bad;
  float* xn_pos;
  uint32_t* list;
  uint32_t* list_count;
  unsigned long long* lkey;
  float* lxn;
};

template <bool IP>
void launch_exact(eb_engine* e, const Top1Args& a, long c0, long m, const ExactScratch& S) {
  unsigned long long* counters = e->counters();
  // pair_count and list_count were zeroed by the screen; k_collect zeroes bad.
  const unsigned rgrid = (unsigned)((m + 255) / 256);
  launch_pdl(e, k_collect<IP>, rgrid, 256, 0, c0, m, (uint32_t)a.k, S.nl, S.cand, S.cand_cnt, S.cand_thr,
                                              S.pairs, S.pair_count, S.rkey, S.list, S.list_count,
                                              S.lkey, S.bad, counters, e->d_status);
  EB_LAUNCH("screen collect");
  // The pair count is known on the device only: persistent blocks stride over it.
  const unsigned pgrid = (unsigned)e->num_sms;
  if (a.d % EX_COLS == 0) {
    launch_pairs<IP>(e, m, a.x, (int)a.d, a.ids, c0, a.c, a.cnorm, a.xnorm, S.pairs,
                     S.pair_count, (uint32_t)a.k, S.rkey, S.xn_pos, S.bad, nullptr);
  } else {
    launch_pdl(e, k_pairs_plain<IP>, pgrid * 4, 128, 0, a.x, (int)a.d, a.ids, c0, a.c, a.cnorm, a.xnorm, S.pairs, S.pair_count, m,
        (uint32_t)a.k, S.rkey, S.xn_pos, S.bad, e->d_status, nullptr);
  }
  EB_LAUNCH("screen exact chains");
  launch_pdl(e, k_finish<IP>, rgrid, 256, 0, a.ids, c0, m, a.xnorm, S.xn_pos, S.rkey, S.bad,
                                             a.labels, a.scores, S.list, S.list_count, S.lkey,
                                             counters);
  EB_LAUNCH("screen finish");
  // The list's length is known on the device only: a grid of a few blocks per
  // SM strides over its (row, centroid block) items; an empty list costs two
  // short launches.
  const long kch = ((long)a.k + LS_C - 1) / LS_C;
  const unsigned lgrid = (unsigned)std::min<long>(m * kch, (long)e->num_sms * 3);
  set_list_smem<IP>(e->device);
  launch_pdl(e, k_list<IP>, lgrid, LS_C, LS_SMEM, a.x, (long)a.n, (int)a.d, a.ids, a.c, a.cnorm,
                                                 (long)a.k, S.list, S.list_count, S.lkey,
                                                 a.xnorm, S.lxn, e->d_status);
  EB_LAUNCH("screen exact list");
  launch_pdl(e, k_list_finish<IP>, (unsigned)std::min<long>((m + 255) / 256, e->num_sms), 256, 0, a.x, (long)a.n, (int)a.d, a.ids, S.list, S.list_count, S.lkey, a.xnorm, S.lxn, a.labels,
      a.scores);
  EB_LAUNCH("screen exact list finish");
}

}  // namespace

namespace {

// The split FP16 bound coefficients of the header comment for this d, with
// 1% slack.
void screen_bound(size_t d, float& e_rel, float& e_abs, float& e_min) {
  const double dd = (double)d;
  const double u24 = std::ldexp(1.0, -24);
  const double gamma_d = dd * u24 / (1.0 - dd * u24);
  e_rel = (float)((3.0 * std::ldexp(1.0, -22) + dd * std::ldexp(1.0, -21) * (1.0 + std::ldexp(1.0, -9)) +
                   dd * std::ldexp(1.0, -30) + std::ldexp(1.0, -23) + gamma_d) *
                  1.01);
  e_abs = (float)(std::ldexp(1.0, -23) * std::sqrt(dd) * 1.01);
  e_min = (float)(dd * std::ldexp(1.0, -48));
}


// The fixed-point screen's bound coefficients for this d, with 1% slack, in
// the integer units of the digits (x' = x xsc, c' = c csc real, v = rint(fl(x')),
// w = rint(fl(c')) with |x' - v|, |c' - w| <= r = 0.502; the MMAs sum
// 65536 hi.hi + 256 (hi.lo + lo.hi) exactly and drop L = sum lo.lo):
//   rounding to integers:  |sum x'c' - sum v w| <= r (|c'|_1 + |v|_1)
//                          <= r sqrt(d) (|x'| + |c'|) + r^2 d
//   dropped products:      |L| <= |x lo| |c lo|                      (e_lo)
//   the epilogue's value a = hi.hi + floor((hi.lo + lo.hi) / 256) in units
//   of 65536: the floor loses less than one unit (65536), and the FP32
//   conversion of a (exact below 2^24) at most 2^-24 65536 |a| <=
//   2^-23 (65536 |hi.hi| + 256 |hi.lo + lo.hi|), where
//   65536 |hi.hi| <= (|x'| + 128.5 sqrt(d)) (|c'| + 128.5 sqrt(d)) and
//   256 |hi.lo + lo.hi| <= 128 sqrt(d) (|x'| + |c'|) + 32896 d:
//                          65536 + 2^-22 (|x'| + 160 sqrt(d)) (|c'| + 160 sqrt(d))
//   the FP32 chain:        gamma_d sum|x' c'| <= gamma_d |x'| |c'|
void screen_bound_q8(size_t d, float& e_rel, float& e_abs, float& e_min, float& e_lo) {
  const double dd = (double)d, sd = std::sqrt(dd);
  const double u24 = std::ldexp(1.0, -24), u22 = std::ldexp(1.0, -22);
  const double gamma_d = dd * u24 / (1.0 - dd * u24);
  e_rel = (float)((gamma_d + u22) * 1.01);
  const double rr = 0.502;
  e_abs = (float)((rr * sd + u22 * 160.0 * sd) * 1.01);
  e_min = (float)((rr * rr * dd + u22 * 160.0 * 160.0 * dd + 65536.0) * 1.01);
  e_lo = 1.01f;
}

// A fresh generation of the centroid summary words.
uint32_t next_gen(eb_engine* e, unsigned long long* cinfo) {
  if (++e->cinfo_gen == 0) {  // wrapped: older tags could compare higher
    EB_CUDA(cudaMemsetAsync(cinfo, 0, 4 * sizeof(unsigned long long), e->stream));
    e->cinfo_gen = 1;
  }
  return e->cinfo_gen;
}

// The fixed-point copy of k rows of c under summary generation gen (with
// `summarise`, the summary is made first).
void convert_with_q8(eb_engine* e, const float* c, size_t k, size_t d, size_t dp8,
                     unsigned long long* cinfo, uint32_t gen, bool summarise, int8_t* ch,
                     int8_t* cl) {
  if (summarise) {
    launch_pdl(e, k_cent_max, (unsigned)((k + 1) / 2), 64, 0, c, (long)k, (int)d, cinfo, gen);
    EB_LAUNCH("screen centroid max");
  }
  launch_pdl(e, k_cent_conv_q8, (unsigned)((k + 1) / 2), 64, 0, c, (long)k, (int)d, (int)dp8,
             cinfo, gen, ch, cl);
  EB_LAUNCH("screen centroid fixed-point copy");
}

// The scaled split FP16 copy of k rows of c (centroids, or data rows playing
// them) and their summary under a new generation, which is returned.
uint32_t convert_centroids(eb_engine* e, const float* c, size_t k, size_t d, size_t dp,
                           unsigned long long* cinfo, __half* ch, __half* cl) {
  const uint32_t gen = next_gen(e, cinfo);
  launch_pdl(e, k_cent_max, (unsigned)((k + 1) / 2), 64, 0, c, (long)k, (int)d, cinfo, gen);
  EB_LAUNCH("screen centroid max");
  launch_pdl(e, k_cent_conv, (unsigned)((k + 1) / 2), 64, 0, c, (long)k, (int)d, (int)dp, cinfo,
             gen, ch, cl);
  EB_LAUNCH("screen centroid convert");
  return gen;
}

}  // namespace

// Parts per row tile: the count (1, 2 or 4, at most the centroid tiles) that
// minimises the screen's length in centroid-tile times, waves of units times
// tiles per part (a unit per SM at a time). More parts mean more candidate
// lists per row for the collect step (two per part), so a larger count is
// taken only when it shortens the screen by a tenth or more. With many row
// tiles every SM is busy at one part; a slice of a few dozen row tiles (a
// training batch split over GPUs) spreads each row tile's centroid tiles over
// several SMs.
int screen_parts(size_t rtiles, int ntiles, int sms) {
  int best = 1;
  size_t best_t = (size_t)-1;
  for (int p = 1; p <= MAX_PARTS && p <= ntiles; p *= 2) {
    const int tpp = (ntiles + p - 1) / p;
    if ((ntiles + tpp - 1) / tpp != p) continue;  // a part would be empty
    const size_t t = (rtiles * (size_t)p + (size_t)sms - 1) / (size_t)sms * (size_t)tpp;
    if (best_t == (size_t)-1 || 10 * t <= 9 * best_t) {
      best_t = t;
      best = p;
    }
  }
  return best;
}

size_t screen_tile_times(size_t rows, size_t k, int sms) {
  const size_t rtiles = (rows + BM - 1) / BM;
  const int ntiles = (int)((k + BN - 1) / BN);
  const int p = screen_parts(rtiles, ntiles, sms);
  const size_t tpp = (size_t)((ntiles + p - 1) / p);
  return (rtiles * (size_t)p + (size_t)sms - 1) / (size_t)sms * tpp;
}

unsigned long long* screen_summary_words(eb_engine* e) {
  return e->scratch_get<unsigned long long>("tc_cinfo", 4, true);
}

uint32_t screen_next_summary_gen(eb_engine* e) { return next_gen(e, screen_summary_words(e)); }

// The split FP16 copy of a bound data set (n x d rows x, buffer xbuf), made
// on first use and kept until the buffer is written or freed; null when xbuf
// is not a bound set of that shape or there is no room for the copy.
Fp16Copy* bound_copy(eb_engine* e, eb_buf* xbuf, const float* x, size_t n, size_t d) {
  if (!xbuf || xbuf->d != d || xbuf->len != n * d) return nullptr;
  const size_t dp = (d + BKH - 1) / BKH * BKH;
  const unsigned wpb = 8;
  if (xbuf->f16 && xbuf->f16->version != xbuf->version) drop_f16(xbuf);
  if (!xbuf->f16) {
    auto* f = new Fp16Copy;
    f->n = n;
    f->d = d;
    f->version = xbuf->version;
    f->stream = e->stream;
    const size_t cells = std::max<size_t>(n * dp, 8);
    cudaError_t st = cudaMallocAsync(&f->xh, cells * 2, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xl, cells * 2, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xexp, std::max<size_t>(n, 1) * 4, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xnrm, std::max<size_t>(n, 1) * 4, e->stream);
    e->device_allocs += 4;
    xbuf->f16 = f;
    if (st != cudaSuccess) {
      free_copy(f);  // no room for the copy: convert per pass instead
      xbuf->f16 = nullptr;
      cudaGetLastError();
    } else if (n) {
      launch_pdl(e, k_prep_rows, (unsigned)((n + wpb - 1) / wpb), wpb * 32, 0, x, (long)n,
                 (int)d, (int)dp, nullptr, 0, (long)n, f->xh, f->xl, f->xexp, f->xnrm,
                 e->d_status);
      EB_LAUNCH("screen copy of bound rows");
    }
  }
  return xbuf->f16;
}

// The fixed-point copy of a bound data set, made on first use and kept until
// the buffer is written or freed; null when xbuf is not a bound set of that
// shape or there is no room for the copy.
Q8Copy* bound_copy_q8(eb_engine* e, eb_buf* xbuf, const float* x, size_t n, size_t d) {
  if (!xbuf || xbuf->d != d || xbuf->len != n * d) return nullptr;
  const size_t dp8 = (d + BK8 - 1) / BK8 * BK8;
  const unsigned wpb = 8;
  if (xbuf->q8 && xbuf->q8->version != xbuf->version) drop_f16(xbuf);
  if (!xbuf->q8) {
    auto* f = new Q8Copy;
    f->n = n;
    f->d = d;
    f->version = xbuf->version;
    f->stream = e->stream;
    const size_t cells = std::max<size_t>(n * dp8, 64);
    const size_t rows = std::max<size_t>(n, 1);
    cudaError_t st = cudaMallocAsync(&f->xh, cells, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xl, cells, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xscl, rows * 4, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xnrm, rows * 4, e->stream);
    if (st == cudaSuccess) st = cudaMallocAsync(&f->xlo, rows * 4, e->stream);
    e->device_allocs += 5;
    xbuf->q8 = f;
    if (st != cudaSuccess) {
      free_q8(f);  // no room for the copy: convert per pass instead
      xbuf->q8 = nullptr;
      cudaGetLastError();
    } else if (n) {
      launch_pdl(e, k_prep_rows_q8, (unsigned)((n + wpb - 1) / wpb), wpb * 32, 0, x, (long)n,
                 (int)d, (int)dp8, nullptr, 0L, (long)n, f->xh, f->xl, f->xscl, f->xnrm, f->xlo,
                 e->d_status);
      EB_LAUNCH("screen fixed-point copy of bound rows");
    }
  }
  return xbuf->q8;
}

bool top1_screen_supported(eb_engine* e, const Top1Args& a) {
  if (e->screen_mode == 0) return false;
  if (a.d > 16384 || a.k > 0x7FFFFFFF) return false;
  if (e->screen_mode == 2) return true;
  return a.k >= 64 && a.r1 - a.r0 >= 128 && a.d >= 16;
}

void top1_screen(eb_engine* e, const Top1Args& a, eb_buf* xbuf) {
  const size_t d = a.d, k = a.k;
  const size_t dp = (d + BK8 - 1) / BK8 * BK8;  // bytes of a fixed-point row
  const size_t m_all = a.r1 - a.r0;
  // Rows per pass: the call split into equal passes of at most twelve
  // 128-row tiles per SM (a C2 assign is one pass), so that each persistent
  // CTA keeps its operand ring running across tiles and the exact stage runs
  // once per pass.
  const size_t wave = (size_t)e->num_sms * BM;
  const size_t max_chunk = PASS_WAVES_TOP1 * wave;
  const size_t npass = (m_all + max_chunk - 1) / max_chunk;
  const size_t chunk =
      std::min(m_all, ((m_all + npass - 1) / std::max<size_t>(npass, 1) + BM - 1) / BM * BM);
  const bool ip = a.metric == EB_IP;

  float e_rel, e_abs, e_min, e_lo;
  screen_bound_q8(d, e_rel, e_abs, e_min, e_lo);

  // Centroids: one shift, fixed-point copy (kept from the last call when the
  // caller says the centroids are unchanged).
  unsigned long long* cinfo = e->scratch_get<unsigned long long>("tc_cinfo", 4, true);
  int8_t* ch = e->scratch_get<int8_t>("tc_ch8", k * dp);
  int8_t* cl = e->scratch_get<int8_t>("tc_cl8", k * dp);
  const unsigned wpb = 8;
  uint32_t cgen = e->cinfo_gen;
  if (!a.centroids_ready) {
    if (a.summary_gen && a.summary_gen == e->cinfo_gen) {
      convert_with_q8(e, a.c, k, d, dp, cinfo, a.summary_gen, false, ch, cl);
    } else {
      cgen = next_gen(e, cinfo);
      convert_with_q8(e, a.c, k, d, dp, cinfo, cgen, true, ch, cl);
    }
  }
  const CUtensorMap mapBh = make_map_q8(ch, k, dp, BN);
  const CUtensorMap mapBl = make_map_q8(cl, k, dp, BN);

  int8_t* xh = e->scratch_get<int8_t>("tc_xh8", chunk * dp);
  int8_t* xl = e->scratch_get<int8_t>("tc_xl8", chunk * dp);
  float* xscl = e->scratch_get<float>("tc_xscl", chunk);
  float* xnrm = e->scratch_get<float>("tc_xnrm", chunk);
  float* xlo = e->scratch_get<float>("tc_xlo", chunk);
  // Parts per row tile for each pass (the pass's row tiles decide them).
  const int ntiles = (int)((k + BN - 1) / BN);
  int max_parts = 1;
  for (size_t c0 = a.r0; c0 < a.r1; c0 += chunk)
    max_parts = std::max(max_parts, screen_parts((std::min(chunk, a.r1 - c0) + BM - 1) / BM,
                                                 ntiles, e->num_sms));
  uint2* cand = e->scratch_get<uint2>("tc_cand", 2 * (size_t)max_parts * chunk * CAP);
  uint32_t* cand_cnt = e->scratch_get<uint32_t>("tc_cnt", 2 * (size_t)max_parts * chunk);
  float* cand_thr = e->scratch_get<float>("tc_thr", 2 * (size_t)max_parts * chunk);
  uint32_t* list = e->scratch_get<uint32_t>("tc_list", chunk);
  uint32_t* list_count = e->scratch_get<uint32_t>("tc_list_count", 4);
  uint2* pairs = e->scratch_get<uint2>("tc_pairs", chunk * SURV);
  uint32_t* pair_count = e->scratch_get<uint32_t>("tc_pair_count", 4);
  unsigned long long* rkey = e->scratch_get<unsigned long long>("tc_rkey", chunk);
  uint32_t* bad = e->scratch_get<uint32_t>("tc_bad", chunk);
  float* xn_pos = e->scratch_get<float>("tc_xn_pos", chunk);
  unsigned long long* lkey = e->scratch_get<unsigned long long>("tc_lkey", chunk);
  float* lxn = e->scratch_get<float>("tc_lxn", chunk);
  ExactScratch S{1, cand, cand_cnt, cand_thr, pairs, pair_count, rkey, bad, xn_pos, list,
                 list_count, lkey, lxn};

  ScreenParams P{};
  P.k = (int)k;
  P.kblocks = (int)(dp / BK8);
  P.ntiles = ntiles;
  P.cn = a.cnorm;
  P.cinfo = cinfo;
  P.cgen = cgen;
  P.e_rel = e_rel;
  P.e_abs = e_abs;
  P.e_min = e_min;
  P.e_lo = e_lo;
  P.cand = cand;
  P.cand_cnt = cand_cnt;
  P.cand_thr = cand_thr;
  P.status = e->d_status;
  P.zero0 = pair_count;
  P.zero1 = list_count;
  P.dead_wait = e->screen_dead_wait;

  // A bound data set keeps its fixed-point copy across calls (training
  // steps, repeated assigns): converted once, then read in place or gathered
  // by id.
  Q8Copy* cache = bound_copy_q8(e, xbuf, a.x, a.n, d);

  for (size_t c0 = a.r0; c0 < a.r1; c0 += chunk) {
    const size_t m = std::min(chunk, a.r1 - c0);
    const int8_t *ah = xh, *al = xl;
    if (cache && !a.ids) {
      // Dense rows of the bound set: the screen reads the cached copy in place.
      ah = cache->xh + c0 * dp;
      al = cache->xl + c0 * dp;
      P.xscl = cache->xscl + c0;
      P.xnrm = cache->xnrm + c0;
      P.xlo = cache->xlo + c0;
    } else if (cache) {
      launch_pdl(e, k_gather_rows_q8, (unsigned)((m + wpb - 1) / wpb), wpb * 32, 0, cache->xh,
                 cache->xl, cache->xscl, cache->xnrm, cache->xlo, (long)a.n, (int)dp, a.ids,
                 (long)c0, (long)m, xh, xl, xscl, xnrm, xlo, e->d_status);
      EB_LAUNCH("screen row gather");
      P.xscl = xscl;
      P.xnrm = xnrm;
      P.xlo = xlo;
    } else {
      launch_pdl(e, k_prep_rows_q8, (unsigned)((m + wpb - 1) / wpb), wpb * 32, 0, a.x, (long)a.n,
                 (int)d, (int)dp, a.ids, (long)c0, (long)m, xh, xl, xscl, xnrm, xlo,
                 e->d_status);
      EB_LAUNCH("screen row prep");
      P.xscl = xscl;
      P.xnrm = xnrm;
      P.xlo = xlo;
    }
    const CUtensorMap mapAh = make_map_q8(ah, m, dp, BM);
    const CUtensorMap mapAl = make_map_q8(al, m, dp, BM);
    P.m = (long)m;
    const size_t rtiles = (m + BM - 1) / BM;
    P.parts = screen_parts(rtiles, ntiles, e->num_sms);
    P.tpp = (ntiles + P.parts - 1) / P.parts;
    P.units = (int)(rtiles * P.parts);
    S.nl = 2 * P.parts;
    // Persistent: at most one CTA per SM, each looping over work units.
    const unsigned grid = (unsigned)std::min<size_t>((size_t)P.units, (size_t)e->num_sms);
    cudaEvent_t ev_end = nullptr;
    if (e->time_screen) {
      if (e->screen_ev_used == e->screen_ev.size()) {
        cudaEvent_t a, b;
        EB_CUDA(cudaEventCreate(&a));
        EB_CUDA(cudaEventCreate(&b));
        e->screen_ev.emplace_back(a, b);
        e->screen_ev_rows.push_back(0);
      }
      const size_t u = e->screen_ev_used++;
      e->screen_ev_rows[u] = m;
      EB_CUDA(cudaEventRecord(e->screen_ev[u].first, e->stream));
      ev_end = e->screen_ev[u].second;
    }
    if (ip)
      launch_screen<true, false, false, true>(e, grid, mapAh, mapAl, mapBh, mapBl, P);
    else
      launch_screen<false, false, false, true>(e, grid, mapAh, mapAl, mapBh, mapBl, P);
    EB_LAUNCH("screen");
    P.dead_wait = e->screen_dead_wait = 0;  // one launch only
    if (ev_end) EB_CUDA(cudaEventRecord(ev_end, e->stream));
    if (ip)
      launch_exact<true>(e, a, (long)c0, (long)m, S);
    else
      launch_exact<false>(e, a, (long)c0, (long)m, S);
  }
  e->stats.screened_rows += m_all;
}


// Top-kk by inner product on the tensor cores: the screen in top-k mode keeps
// every column within 2e of each row's screened kk-th best (a column of the
// exact top kk cannot lie further below it), the exact FP32 chains score
// those candidates, and each row takes its best kk by (larger score, then
// lower id); rows with too many candidates are scanned exactly in full.
bool topk_screen(eb_engine* e, const float* q, size_t m, const float* data, size_t n, size_t d,
                 size_t kk, bool exclude_self, uint32_t* ids, float* sims, size_t id0) {
  if (e->screen_mode == 0 || d > 16384 || n > 0x7FFFFFFFull || kk > (size_t)KMAX) return false;
  if (e->screen_mode == 1 && (n < 256 || m < 128 || d < 16)) return false;
  const size_t dp = (d + BK8 - 1) / BK8 * BK8;  // bytes of a fixed-point row
  const size_t wave = (size_t)e->num_sms * BM;
  const size_t chunk = std::min(m, PASS_WAVES * wave);
  float e_rel, e_abs, e_min, e_lo;
  screen_bound_q8(d, e_rel, e_abs, e_min, e_lo);

  // The data rows play the centroids: one scale, fixed-point copy (the two
  // int8 digits of each value, as in the top-1 screen).
  unsigned long long* cinfo = e->scratch_get<unsigned long long>("tc_cinfo", 4, true);
  int8_t* ch = e->scratch_get<int8_t>("tc_ch8", n * dp);
  int8_t* cl = e->scratch_get<int8_t>("tc_cl8", n * dp);
  const uint32_t cgen = next_gen(e, cinfo);
  convert_with_q8(e, data, n, d, dp, cinfo, cgen, true, ch, cl);
  const CUtensorMap mapBh = make_map_q8(ch, n, dp, BN);
  const CUtensorMap mapBl = make_map_q8(cl, n, dp, BN);

  const unsigned wpb = 8;
  int8_t* xh = e->scratch_get<int8_t>("tc_xh8", chunk * dp);
  int8_t* xl = e->scratch_get<int8_t>("tc_xl8", chunk * dp);
  float* xscl = e->scratch_get<float>("tc_xscl", chunk);
  float* xnrm = e->scratch_get<float>("tc_xnrm", chunk);
  float* xlo = e->scratch_get<float>("tc_xlo", chunk);
  uint2* cand = e->scratch_get<uint2>("tc_cand", 2 * chunk * CAP_TOPK);
  uint32_t* cand_cnt = e->scratch_get<uint32_t>("tc_cnt", 2 * chunk);
  float* cand_thr = e->scratch_get<float>("tc_thr", 2 * chunk);
  float* kvals = e->scratch_get<float>("tk_kvals", 2 * chunk * KMAX);
  float* roff = e->scratch_get<float>("tk_roff", chunk);
  uint2* pairs = e->scratch_get<uint2>("tc_pairs", chunk * SURV);
  float* pval = e->scratch_get<float>("tk_pval", chunk * SURV);
  uint32_t* pair_count = e->scratch_get<uint32_t>("tc_pair_count", 4);
  uint32_t* pstart = e->scratch_get<uint32_t>("tk_pstart", chunk);
  uint32_t* pcnt = e->scratch_get<uint32_t>("tk_pcnt", chunk);
  uint32_t* list = e->scratch_get<uint32_t>("tc_list", chunk);
  uint32_t* list_count = e->scratch_get<uint32_t>("tc_list_count", 4);
  uint32_t* h_list_count = e->h_status + 1;  // pinned word beside the status mirror
  unsigned long long* counters = e->counters();

  ScreenParams P{};
  P.k = (int)n;
  P.kblocks = (int)(dp / BK8);
  P.ntiles = (int)((n + BN - 1) / BN);
  P.parts = 1;  // the top-k collect merges the two halves' best-kk lists
  P.tpp = P.ntiles;
  P.cn = nullptr;
  P.cinfo = cinfo;
  P.cgen = cgen;
  P.e_rel = e_rel;
  P.e_abs = e_abs;
  P.e_min = e_min;
  P.e_lo = e_lo;
  P.cand = cand;
  P.cand_cnt = cand_cnt;
  P.cand_thr = cand_thr;
  P.status = e->d_status;
  P.zero0 = pair_count;
  P.zero1 = list_count;
  P.kk = (int)kk;
  P.exclude_self = exclude_self ? 1 : 0;
  P.col_gid0 = (long)id0;
  P.kvals = kvals;
  P.roff = roff;

  for (size_t c0 = 0; c0 < m; c0 += chunk) {
    const size_t mc = std::min(chunk, m - c0);
    launch_pdl(e, k_prep_rows_q8, (unsigned)((mc + wpb - 1) / wpb), wpb * 32, 0, q, (long)m,
               (int)d, (int)dp, nullptr, (long)c0, (long)mc, xh, xl, xscl, xnrm, xlo,
               e->d_status);
    EB_LAUNCH("topk query prep");
    const CUtensorMap mapAh = make_map_q8(xh, mc, dp, BM);
    const CUtensorMap mapAl = make_map_q8(xl, mc, dp, BM);
    P.m = (long)mc;
    P.units = (int)((mc + BM - 1) / BM);
    P.xscl = xscl;
    P.xnrm = xnrm;
    P.xlo = xlo;
    P.row_gid0 = (long)c0;
    const unsigned grid = (unsigned)std::min<size_t>((mc + BM - 1) / BM, (size_t)e->num_sms);
    launch_screen<true, true, false, true>(e, grid, mapAh, mapAl, mapBh, mapBl, P);
    EB_LAUNCH("topk screen");
    const unsigned rgrid = (unsigned)((mc + 255) / 256);
    launch_pdl(e, k_collect_topk, rgrid, 256, 0, (long)c0, (long)mc, (uint32_t)n, (int)kk, cand,
                                                 cand_cnt, kvals, roff, pairs, pair_count, pstart,
                                                 pcnt, list, list_count, counters, e->d_status);
    EB_LAUNCH("topk collect");
    const unsigned pgrid = (unsigned)e->num_sms;
    if (d % EX_COLS == 0) {
      launch_pairs<true>(e, (long)mc, q, (int)d, nullptr, (long)c0, data, nullptr, nullptr, pairs,
                         pair_count, (uint32_t)n, nullptr, nullptr, nullptr, pval);
    } else {
      launch_pdl(e, k_pairs_plain<true>, pgrid * 4, 128, 0, q, (int)d, nullptr, (long)c0, data, nullptr, nullptr, pairs, pair_count, (long)mc,
          (uint32_t)n, nullptr, nullptr, nullptr, e->d_status, pval);
    }
    EB_LAUNCH("topk exact chains");
    launch_pdl(e, k_topk_finish, rgrid, 256, 0, (long)c0, (long)mc, (int)kk, (uint32_t)id0,
                                                pstart, pcnt, pairs, pval, ids, sims);
    EB_LAUNCH("topk finish");
    // Rows of the full scan: their count comes to the host (this call ends
    // with a copy to the host anyway), then a chunked exact scan.
    EB_CUDA(cudaMemcpyAsync(h_list_count, list_count, 4, cudaMemcpyDeviceToHost, e->stream));
    EB_CUDA(cudaStreamSynchronize(e->stream));
    const size_t L = *h_list_count;
    if (L) {
      float* gq = e->scratch_get<float>("tk_gq", L * d);
      uint32_t* tids = e->scratch_get<uint32_t>("tk_tids", L * kk);
      float* tsims = e->scratch_get<float>("tk_tsims", L * kk);
      const unsigned gx = (unsigned)std::min<size_t>(L, 65535);
      const unsigned gy = (unsigned)((L + gx - 1) / gx);
      launch_pdl(e, k_gather_queries, dim3(gx, gy), 128, 0, q, (int)d, list, (long)L, gq);
      EB_LAUNCH("topk gather");
      topk_exact_device(e, gq, L, list, data, n, d, kk, exclude_self, tids, tsims, id0);
      launch_pdl(e, k_scatter_topk, (unsigned)((L * kk + 255) / 256), 256, 0, list, (long)L, (int)kk, tids, tsims, ids, sims);
      EB_LAUNCH("topk scatter");
    }
  }
  e->stats.screened_rows += m;
  return true;
}

// The internal scores' n x k_eff product on the tensor cores (the screen in
// product mode): for each row i of x (n x d, f32 on the device) with own
// column slot[labels[i]], best_out[i] = the column s != own of the largest
// x_i . c_s * inv[s], from the split FP16 products (xh ch + xh cl + xl ch,
// FP32 accumulation); 0xFFFFFFFF when k = 1, 0xFFFFFFFE for rows the screen
// could not score (non-finite values, a wait that gave up). The bound set's
// split copy is read in place when xbuf holds one.
void screen_products(eb_engine* e, const float* x, size_t n, size_t d, eb_buf* xbuf,
                     const uint32_t* labels, const uint32_t* slot, const float* c,
                     const float* inv, size_t k, uint32_t* best_out) {
  if (n == 0) return;
  const size_t dp = (d + BKH - 1) / BKH * BKH;
  const size_t wave = (size_t)e->num_sms * BM;
  const size_t chunk = std::min(n, PASS_WAVES * wave);
  float e_rel, e_abs, e_min;
  screen_bound(d, e_rel, e_abs, e_min);
  unsigned long long* cinfo = e->scratch_get<unsigned long long>("tc_cinfo", 4, true);
  __half* ch = e->scratch_get<__half>("tc_ch", k * dp);
  __half* cl = e->scratch_get<__half>("tc_cl", k * dp);
  const uint32_t cgen = convert_centroids(e, c, k, d, dp, cinfo, ch, cl);
  const CUtensorMap mapBh = make_map(ch, k, dp, BN);
  const CUtensorMap mapBl = make_map(cl, k, dp, BN);
  const int ntiles = (int)((k + BN - 1) / BN);
  int max_parts = 1;
  for (size_t c0 = 0; c0 < n; c0 += chunk)
    max_parts = std::max(max_parts, screen_parts((std::min(chunk, n - c0) + BM - 1) / BM,
                                                 ntiles, e->num_sms));
  const unsigned wpb = 8;
  __half* xh = e->scratch_get<__half>("tc_xh", chunk * dp);
  __half* xl = e->scratch_get<__half>("tc_xl", chunk * dp);
  int* xexp = e->scratch_get<int>("tc_xexp", chunk);
  float* xnrm = e->scratch_get<float>("tc_xnrm", chunk);
  float* pmax = e->scratch_get<float>("pr_max", 2 * (size_t)max_parts * chunk);
  uint32_t* pcol = e->scratch_get<uint32_t>("pr_col", 2 * (size_t)max_parts * chunk);
  // A bound data set keeps its split FP16 copy (made by the first product
  // call, kept until the buffer is written or freed): later calls on it,
  // such as a sweep's internal scores, read it in place.
  Fp16Copy* cache = bound_copy(e, xbuf, x, n, d);

  ScreenParams P{};
  P.k = (int)k;
  P.kblocks = (int)(dp / BKH);
  P.ntiles = ntiles;
  P.cinfo = cinfo;
  P.cgen = cgen;
  P.e_rel = e_rel;
  P.e_abs = e_abs;
  P.e_min = e_min;
  P.status = e->d_status;
  P.plabels = labels;
  P.pslot = slot;
  P.pinv = inv;
  P.pmax = pmax;
  P.pcol = pcol;
  for (size_t c0 = 0; c0 < n; c0 += chunk) {
    const size_t m = std::min(chunk, n - c0);
    const __half *ah = xh, *al = xl;
    const int* pe = xexp;
    if (cache) {
      ah = cache->xh + c0 * dp;
      al = cache->xl + c0 * dp;
      pe = cache->xexp + c0;
      P.xexp = pe;
      P.xnrm = cache->xnrm + c0;
    } else {
      launch_pdl(e, k_prep_rows, (unsigned)((m + wpb - 1) / wpb), wpb * 32, 0, x, (long)n,
                 (int)d, (int)dp, nullptr, (long)c0, (long)m, xh, xl, xexp, xnrm, e->d_status);
      EB_LAUNCH("product row prep");
      P.xexp = xexp;
      P.xnrm = xnrm;
    }
    const CUtensorMap mapAh = make_map(ah, m, dp, BM);
    const CUtensorMap mapAl = make_map(al, m, dp, BM);
    P.m = (long)m;
    P.prow0 = (long)c0;
    const size_t rtiles = (m + BM - 1) / BM;
    P.parts = screen_parts(rtiles, ntiles, e->num_sms);
    P.tpp = (ntiles + P.parts - 1) / P.parts;
    P.units = (int)(rtiles * P.parts);
    const unsigned grid = (unsigned)std::min<size_t>((size_t)P.units, (size_t)e->num_sms);
    launch_screen<true, false, true>(e, grid, mapAh, mapAl, mapBh, mapBl, P);
    EB_LAUNCH("product screen");
    launch_pdl(e, k_prod_finish, (unsigned)((m + 255) / 256), 256, 0, (long)c0, (long)m,
               2 * P.parts, pe, cinfo, cgen, pmax, pcol, best_out);
    EB_LAUNCH("product finish");
  }
}

}  // namespace eb
