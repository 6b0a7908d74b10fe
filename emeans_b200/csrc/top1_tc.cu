// Exact top-1 on the tensor cores: a tcgen05 FP16 screen, then an exact FP32
// re-score of the few centroids the screen cannot rule out.
//
// The labels and scores are the reference CPU kernel's bit for bit
// (crates/emeans-core/src/assign/fused.rs:12-16: one sequential FMA chain per
// dot, lower id on ties). The screen only decides which centroids get that
// exact chain:
//
// 1. prep: rows and centroids are scaled by powers of two (per row for x, one
//    exponent for all centroids) so that |v| < 2^14, and rounded to FP16.
// 2. screen (tcgen05): a 128-row tile of x against 256-centroid tiles, FP32
//    accumulators in TMEM (two buffers of 256 columns, so the epilogue reads
//    one while the tensor cores fill the other), operands staged by TMA into
//    128B-swizzled shared memory through a 4-stage mbarrier ring. The
//    epilogue (one thread per row) reads each 256-column tile from TMEM twice:
//    first for the tile's best score, which moves the row's running best, then
//    to append every centroid within 2e of that best to the row's candidate
//    list, where e bounds |screen - exact chain| (FP16 rounding of both
//    operands, tensor-core accumulation, the FP32 chain itself). A centroid
//    more than 2e behind the best cannot be the exact winner.
// 3. refine (one warp per row): a precise FP32 dot per candidate with its own
//    error bound (from the computed sum |x_t c_t|) leaves the candidates that
//    could still be the exact best, usually one.
// 4. exact (one thread per row): the exact FMA chain of each survivor; lower
//    id on ties.
// 5. fallback: rows with too many candidates, or non-finite inputs, take the
//    exact SIMT kernel (top1_exact.cu).
//
// Error bound (acc units, operands scaled): with u = 2^-11 and FP16
// subnormals (half-ulp 2^-25),
//   |acc - x'.c'| <= (2^-10 + 2^-22) sum|x'||c'| + 2^-24 (sum|x'| + sum|c'|)
//                    + d 2^-21 sum|x'||c'|        (accumulation, taken loose)
// and the FP32 chain differs from the exact dot by <= gamma_d sum|x c|.
// sum|x'||c'| <= |x'| |c'|, sum|x'| <= sqrt(d) |x'| (Cauchy-Schwarz).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>

#include "engine.h"

namespace eb {

// The FP16 screen copy of a bound data set (its scaled rows, exponents and
// norm bounds), built by the first screened top-1 on the set and kept until
// the buffer is written or freed.
struct Fp16Copy {
  __half* xh = nullptr;  // n x dp
  int* xexp = nullptr;
  float* xnrm = nullptr;
  size_t n = 0, d = 0;
  uint64_t version = 0;
  cudaStream_t stream = nullptr;
};

void drop_f16(eb_buf* b) {
  if (b && b->f16) {
    Fp16Copy* f = b->f16;
    cudaFreeAsync(f->xh, f->stream);
    cudaFreeAsync(f->xexp, f->stream);
    cudaFreeAsync(f->xnrm, f->stream);
    delete f;
    b->f16 = nullptr;
  }
}

namespace {

constexpr int BM = 128;          // rows per CTA (TMEM lanes)
constexpr int BN = 256;          // centroids per tile (TMEM columns per buffer)
constexpr int BKH = 64;          // FP16 columns per k-block: one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKH * 2;
constexpr int B_BYTES = BN * BKH * 2;
constexpr int CAP = 128;         // per-row candidate list capacity
constexpr int NTHREADS = 192;    // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t FALLBACK = 0xFFFFFFFFu;
constexpr int XEXP_BAD = INT_MIN;  // row with a non-finite value
constexpr size_t PASS_WAVES = 8;  // row tiles per SM in one pass
constexpr uint64_t WAIT_NS = 2000000000ull;  // bounded waits: 2 s

// Operand ring, then 256 B of barriers / TMEM slot / flags, then per epilogue
// warp two tiles of centroid norms.
constexpr size_t SMEM_BYTES =
    1024 /* alignment slack */ + STAGES * (A_BYTES + B_BYTES) + 256 + 4 * 2 * BN * sizeof(float);

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
  uint64_t t0 = now_ns();
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

// K-major operand tile with 128-byte rows, 128B swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
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

// 64 consecutive FP32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]),
        "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]),
        "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]),
        "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Screened scores of 64 columns of this thread's row, `lim` of them real
// (lim >= 64: all): the raw accumulator (IP), or the key cn_j - 2 f acc_j with
// one rounding (L2), with the norms read from shared memory. Columns past k
// score -inf (IP) / +inf (L2), so they never win or enter.
template <bool IP>
__device__ __forceinline__ void group_scores(uint32_t taddr, const float* cns, float m2f, int lim,
                                             float (&s)[64]) {
  uint32_t v[64];
  tmem_ld64(taddr, v);
  if (IP) {
#pragma unroll
    for (int j = 0; j < 64; j++) s[j] = __uint_as_float(v[j]);
  } else {
    const float4* c4 = reinterpret_cast<const float4*>(cns);
#pragma unroll
    for (int j = 0; j < 64; j += 4) {
      const float4 c = c4[j / 4];
      s[j] = __fmaf_rn(m2f, __uint_as_float(v[j]), c.x);
      s[j + 1] = __fmaf_rn(m2f, __uint_as_float(v[j + 1]), c.y);
      s[j + 2] = __fmaf_rn(m2f, __uint_as_float(v[j + 2]), c.z);
      s[j + 3] = __fmaf_rn(m2f, __uint_as_float(v[j + 3]), c.w);
    }
  }
  if (lim < 64) {
#pragma unroll
    for (int j = 0; j < 64; j++)
      if (j >= lim) s[j] = IP ? -INFINITY : INFINITY;
  }
}

// Keep only the entries of a row's candidate list still inside the window
// (out of line: it runs only when a list nears its capacity).
template <bool IP>
__device__ __noinline__ uint32_t compact_list(uint2* list, uint32_t cnt, float thr) {
  uint32_t w = 0;
  for (uint32_t e = 0; e < cnt; e++) {
    const uint2 en = list[e];
    const float sv = __uint_as_float(en.y);
    if (IP ? (sv >= thr) : (sv <= thr)) list[w++] = en;
  }
  return w;
}

// ---------------------------------------------------------------- prep kernels

// Scaled FP16 copy of the selected rows (one warp per row), with the row's
// exponent (XEXP_BAD for non-finite rows) and an upper bound on its norm.
__global__ void k_prep_rows(const float* __restrict__ x, long n, int d, int dp,
                            const uint32_t* __restrict__ ids, long p0, long m,
                            __half* __restrict__ xh, int* __restrict__ xexp,
                            float* __restrict__ xnrm, uint32_t* status) {
  long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (i >= m) return;
  long p = p0 + i;
  long row = ids ? (long)ids[p] : p;
  __half* out = xh + i * (long)dp;
  if (row >= n) {
    if (lane == 0) {
      atomicOr(status, ST_BAD_ROW);
      xexp[i] = XEXP_BAD;
      xnrm[i] = 0.0f;
    }
    for (int t = lane; t < dp; t += 32) out[t] = __float2half_rn(0.0f);
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
        __half2 h0 = finite ? __floats2half2_rn(ldexpf(v[u].x, sh), ldexpf(v[u].y, sh))
                            : __floats2half2_rn(0.f, 0.f);
        __half2 h1 = finite ? __floats2half2_rn(ldexpf(v[u].z, sh), ldexpf(v[u].w, sh))
                            : __floats2half2_rn(0.f, 0.f);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(out + 4 * t) = pk;
      }
    }
    for (int t = d + lane; t < dp; t += 32) out[t] = __float2half_rn(0.0f);
  } else {
    for (int t = lane; t < d; t += 32) {
      float v = __ldg(r + t);
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
      float v = t < d ? __ldg(r + t) : 0.0f;
      out[t] = __float2half_rn(finite ? ldexpf(v, sh) : 0.0f);
    }
  }
  if (lane == 0) {
    xexp[i] = finite ? ex : XEXP_BAD;
    // Any-order sum of squares: relative error < d 2^-24; inflate by 2^-9.
    xnrm[i] = finite ? sqrtf(ss) * (1.0f + 1.0f / 512.0f) : 0.0f;
  }
}

// Rows x[ids[p]] of a cached FP16 copy gathered into the pass's staging rows
// (one warp per row, 16-byte copies; dp * 2 bytes is a multiple of 128).
__global__ void k_gather_rows(const __half* __restrict__ src_h, const int* __restrict__ src_e,
                              const float* __restrict__ src_n, long n, int dp,
                              const uint32_t* __restrict__ ids, long p0, long m,
                              __half* __restrict__ xh, int* __restrict__ xexp,
                              float* __restrict__ xnrm, uint32_t* status) {
  const long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= m) return;
  const long row = ids[p0 + i];
  uint4* out = reinterpret_cast<uint4*>(xh + i * (long)dp);
  const int q = dp / 8;
  if (row >= n) {
    for (int t = lane; t < q; t += 32) out[t] = make_uint4(0, 0, 0, 0);
    if (lane == 0) {
      atomicOr(status, ST_BAD_ROW);
      xexp[i] = XEXP_BAD;
      xnrm[i] = 0.0f;
    }
    return;
  }
  const uint4* in = reinterpret_cast<const uint4*>(src_h + row * (long)dp);
  for (int t = lane; t < q; t += 32) out[t] = __ldg(in + t);
  if (lane == 0) {
    xexp[i] = src_e[row];
    xnrm[i] = src_n[row];
  }
}

// Global max |c|, a bound on max |c_j| and a non-finite flag, over all centroids.
// cinfo (u32): [0] bits of max|c|, [1] bits of the norm bound, [2] non-finite flag.
__global__ void k_cent_max(const float* __restrict__ c, long k, int d, uint32_t* cinfo) {
  long j = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (j >= k) return;
  const float* r = c + j * (long)d;
  float mx = 0.0f, ss = 0.0f;
  bool finite = true;
  for (int t = lane; t < d; t += 32) {
    float v = __ldg(r + t);
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
  if (lane == 0) {
    if (!finite) {
      atomicOr(&cinfo[2], 1u);
      return;
    }
    atomicMax(&cinfo[0], __float_as_uint(mx));
    atomicMax(&cinfo[1], __float_as_uint(sqrtf(ss) * (1.0f + 1.0f / 512.0f)));
  }
}

// Scaled FP16 centroids: c' = c 2^(14 - ec), 2^(ec-1) <= max|c| < 2^ec.
__global__ void k_cent_conv(const float* __restrict__ c, long k, int d, int dp,
                            const uint32_t* __restrict__ cinfo, __half* __restrict__ ch) {
  long j = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (j >= k) return;
  int ec = 0;
  frexpf(__uint_as_float(cinfo[0]), &ec);
  int sh = 14 - ec;
  bool bad = cinfo[2] != 0;
  const float* r = c + j * (long)d;
  __half* out = ch + j * (long)dp;
  for (int t = lane; t < dp; t += 32) {
    float v = (t < d && !bad) ? __ldg(r + t) : 0.0f;
    out[t] = __float2half_rn(ldexpf(v, sh));
  }
}

// ---------------------------------------------------------------- the screen

struct ScreenParams {
  long m;              // staging rows in this launch
  int k;
  int kblocks;         // dp / 64
  int ntiles;          // ceil(k / 256)
  int d;
  const int* xexp;     // per staging row
  const float* xnrm;   // per staging row
  const float* cn;     // k squared centroid norms (L2) or null
  const uint32_t* cinfo;
  float e_rel, e_abs, e_min;  // bound coefficients (see the header comment)
  uint2* cand;         // m x CAP (id, screened value bits)
  uint32_t* cand_cnt;  // m: entries in use, or FALLBACK
  float* cand_thr;     // m: the final admission threshold
  uint32_t* status;
};

template <bool IP>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_screen(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             ScreenParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = (uint64_t*)(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* cn_s = (float*)(smem + STAGES * (A_BYTES + B_BYTES) + 256);  // [4 warps][2][BN] (L2)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(mma_done, 1);
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
  const uint32_t tmem = *tmem_slot;
  const int total = P.ntiles * P.kblocks;

  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: per (row tile, centroid tile, k-block), one A box
      // (128 x 64) and one B box (256 x 64). The ring runs on across row tiles.
      int it = 0, issued = 0;
      bool stop = false;
      for (long rt = blockIdx.x; rt * BM < P.m && !stop; rt += gridDim.x) {
        for (int t2 = 0; t2 < total; t2++, it++) {
          const int s = it % STAGES;
          const uint32_t par = ((it / STAGES) & 1) ^ 1;
          if (!mbar_wait(&empty[s], par, abort_flag)) {
            stop = true;
            break;
          }
          const int nt = t2 / P.kblocks, kb = t2 % P.kblocks;
          mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmA, &full[s], kb * BKH, (int)(rt * BM));
          tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * BKH, nt * BN);
          issued = it + 1;
        }
      }
      // No copy may still be landing in shared memory when the CTA exits: wait
      // (bounded) for the last loads issued. On the normal path they have
      // already been consumed and these waits return at once.
      for (int it = issued > STAGES ? issued - STAGES : 0; it < issued; it++) {
        uint64_t t0 = now_ns();
        while (!mbar_try_wait(&full[it % STAGES], (it / STAGES) & 1) && now_ns() - t0 < WAIT_NS) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer; tc counts (row tile, centroid tile) pairs for the TMEM buffers.
      int it = 0, tc = 0;
      bool stop = false;
      for (long rt = blockIdx.x; rt * BM < P.m && !stop; rt += gridDim.x)
      for (int nt = 0; nt < P.ntiles; nt++, tc++) {
        const int a = tc & 1;
        if (!mbar_wait(&tempty[a], ((tc >> 1) & 1) ^ 1, abort_flag)) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(a * BN);
        bool ok = true;
        for (int kb = 0; kb < P.kblocks; kb++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BKH / 16; kk++)
            umma_f16(dcol, umma_desc(a0 + kk * 32), umma_desc(b0 + kk * 32),
                     (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) {
          stop = true;
          break;
        }
        umma_commit(&tfull[a]);
      }
      // Every MMA this thread issued has completed once mma_done flips.
      umma_commit(mma_done);
      uint64_t t0 = now_ns();
      while (!mbar_try_wait(mma_done, 0) && now_ns() - t0 < WAIT_NS) {
      }
    }
  } else {
    // Epilogue: one thread per row of each row tile.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int ec = 0;
    frexpf(__uint_as_float(P.cinfo[0]), &ec);
    const float cmax = __uint_as_float(P.cinfo[1]);
    const bool c_bad = P.cinfo[2] != 0;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    int tc = 0;  // (row tile, centroid tile) pairs, as the MMA issuer counts them
    bool stop = false;
    for (long rt = blockIdx.x; rt * BM < P.m && !stop; rt += gridDim.x) {
    const long i = rt * BM + r;
    const bool live = i < P.m;
    const int ex = live ? P.xexp[i] : XEXP_BAD;
    bool fallback = !live || ex == XEXP_BAD || c_bad;
    const float xn = live ? P.xnrm[i] : 0.0f;
    // |x'| and max |c'| in acc units, and the bound e (acc units).
    const float xs = ldexpf(xn, 14 - (fallback ? 0 : ex));
    const float cs = ldexpf(cmax, 14 - ec);
    const float e_acc = fmaf(P.e_rel * xs, cs, fmaf(P.e_abs, xs + cs, P.e_min));
    float off, m2f = 0.0f;
    if (IP) {
      off = 2.0f * e_acc;
    } else {
      const int fe = ex + ec - 28;
      if (fe < -100 || fe > 100) fallback = true;
      const float f = ldexpf(1.0f, fallback ? 0 : fe);
      m2f = -2.0f * f;
      const float e_key = fmaf(2.0f * f, e_acc, ldexpf(fmaf(cmax, cmax, 2.0f * xn * cmax), -22));
      off = 2.0f * e_key;
    }
    if (!isfinite(off)) fallback = true;
    const bool collect = live && !fallback;
    float best = IP ? -INFINITY : INFINITY;
    float thr = best;
    bool overflow = false;
    uint32_t cnt = 0;  // entries in this row's candidate list
    uint2* row_list = P.cand + (live ? i : 0) * (long)CAP;

    for (int nt = 0; nt < P.ntiles; nt++, tc++) {
      const int a = tc & 1;
      // Warp-uniform: the TMEM loads below are .sync.aligned.
      const bool ready = __all_sync(0xFFFFFFFFu, mbar_wait(&tfull[a], (tc >> 1) & 1, abort_flag));
      if (!ready) {
        stop = true;
        break;
      }
      tc_fence_after();
      const int col0 = nt * BN;
      const uint32_t tbase = lane_base + (uint32_t)(a * BN);
      // This tile's squared centroid norms, staged by each warp for itself (no
      // barrier across warps, so a timed-out wait can never strand another warp).
      float* cns = cn_s + (q * 2 + a) * BN;
      if (!IP) {
#pragma unroll
        for (int u = 0; u < BN / 32; u++) {
          const int c = u * 32 + lane;
          cns[c] = col0 + c < P.k ? __ldg(P.cn + col0 + c) : 0.0f;
        }
        __syncwarp();
      }
      const int ngr = min(BN / 64, (P.k - col0 + 63) / 64);
#pragma unroll 1
      for (int g = 0; g < ngr; g++) {
        // One pass per 64 columns: scores, their best (which moves the
        // threshold first), then every score within the window is appended.
        float s[64];
        group_scores<IP>(tbase + (uint32_t)(g * 64), cns + g * 64, m2f, P.k - (col0 + g * 64), s);
        float gb;
        {
          float t[32];
#pragma unroll
          for (int j = 0; j < 32; j++) t[j] = IP ? fmaxf(s[j], s[j + 32]) : fminf(s[j], s[j + 32]);
#pragma unroll
          for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
            for (int j = 0; j < w2; j++) t[j] = IP ? fmaxf(t[j], t[j + w2]) : fminf(t[j], t[j + w2]);
          gb = t[0];
        }
        if (IP ? (gb > best) : (gb < best)) {
          best = gb;
          thr = IP ? __fsub_rd(best, off) : __fadd_ru(best, off);
        }
        // Straight-line admission mask; the append runs only when it is set.
        uint32_t adm_lo = 0, adm_hi = 0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          adm_lo |= (uint32_t)(IP ? (s[j] >= thr) : (s[j] <= thr)) << j;
          adm_hi |= (uint32_t)(IP ? (s[j + 32] >= thr) : (s[j + 32] <= thr)) << j;
        }
        if (collect && (adm_lo | adm_hi)) {
          if (cnt + 64 > CAP) cnt = compact_list<IP>(row_list, cnt, thr);
          const uint32_t base = (uint32_t)(col0 + g * 64);
#pragma unroll
          for (int j = 0; j < 64; j++) {
            const bool in = ((j < 32 ? adm_lo : adm_hi) >> (j & 31)) & 1u;
            if (in) {
              if (cnt < CAP) row_list[cnt] = make_uint2(base + j, __float_as_uint(s[j]));
              overflow |= cnt >= CAP;
              cnt += cnt < CAP;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
    if (live) {
      const bool ok = collect && !overflow && isfinite(best) && !*abort_flag;
      if (ok) P.cand_thr[i] = thr;
      P.cand_cnt[i] = ok ? cnt : FALLBACK;
    }
    }  // row tiles
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(P.status, ST_WAIT_TIMEOUT);
}

// ---------------------------------------------------------------- exact re-score
//
// Stage 1 (k_refine, one warp per row): each admitted candidate gets a precise
// FP32 dot with the lanes splitting d, plus the sum of |x_t c_t| that bounds
// its error; only candidates that could still be the exact best survive.
// Stage 2 (k_exact, one thread per row): the exact FMA chain of each survivor
// (usually one) gives the label and the bit-exact score.

constexpr int SURV = 8;  // survivors per row kept for the exact chains

template <bool IP>
__device__ __forceinline__ bool better(float v, uint32_t j, float bv, uint32_t bj) {
  if (bj == FALLBACK) return true;
  return IP ? (v > bv || (v == bv && j < bj)) : (v < bv || (v == bv && j < bj));
}

__device__ __forceinline__ void to_list(uint32_t p, uint32_t* list, uint32_t* list_count,
                                        unsigned long long* counters) {
  list[atomicAdd(list_count, 1u)] = p;
  atomicAdd(&counters[1], 1ull);
}

template <bool IP>
__global__ void __launch_bounds__(256) k_refine(
    const float* __restrict__ x, int d, const uint32_t* __restrict__ ids, long p0, long m,
    const float* __restrict__ c, const float* __restrict__ cn, const uint2* __restrict__ cand,
    const uint32_t* __restrict__ cand_cnt, const float* __restrict__ cand_thr, float e2,
    uint2* __restrict__ pairs, uint32_t* __restrict__ pair_count,
    unsigned long long* __restrict__ rkey, uint32_t* __restrict__ list,
    uint32_t* __restrict__ list_count, unsigned long long* __restrict__ counters) {
  __shared__ float pv_s[8][CAP], pe_s[8][CAP];
  __shared__ uint32_t pj_s[8][CAP];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long i = (long)blockIdx.x * 8 + w;
  if (i >= m) return;
  const uint32_t cnt = cand_cnt[i];
  if (cnt == FALLBACK) {
    if (lane == 0) {
      rkey[i] = IP ? 0ull : ~0ull;
      to_list((uint32_t)(p0 + i), list, list_count, counters);
    }
    return;
  }
  const float thr = cand_thr[i];
  const long p = p0 + i;
  const long row = ids ? (long)ids[p] : p;
  const float* xr = x + row * (long)d;
  float* pv = pv_s[w];
  float* pe = pe_s[w];
  uint32_t* pj = pj_s[w];
  int np = 0;
  // The row's x (a float4 per lane per 128 columns) stays in registers for
  // every candidate when d % 4 == 0 and d <= 1024; otherwise it is re-read.
  const bool vec = (d & 3) == 0 && d <= 1024;
  const int q4 = d / 4;
  float4 xv[8];
#pragma unroll
  for (int u = 0; u < 8; u++) {
    const int t = lane + 32 * u;
    xv[u] = (vec && t < q4) ? __ldg(reinterpret_cast<const float4*>(xr) + t)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  uint32_t e = 0;
  while (true) {
    // The next two candidates still inside the final window (the rest were
    // left behind by it), scored together so their loads overlap.
    uint32_t jc[2] = {FALLBACK, FALLBACK};
#pragma unroll
    for (int h = 0; h < 2; h++) {
      while (e < cnt) {
        const uint2 en = cand[i * (long)CAP + e++];
        const float sv = __uint_as_float(en.y);
        if (IP ? sv >= thr : sv <= thr) {
          jc[h] = en.x;
          break;
        }
      }
    }
    if (jc[0] == FALLBACK) break;
    float dot[2] = {0.0f, 0.0f}, ab[2] = {0.0f, 0.0f};
    if (vec) {
      const float4* c40 = reinterpret_cast<const float4*>(c + (long)jc[0] * d);
      const float4* c41 = reinterpret_cast<const float4*>(
          c + (long)(jc[1] == FALLBACK ? jc[0] : jc[1]) * d);
      float4 ca[8], cb[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int t = lane + 32 * u;
        ca[u] = t < q4 ? __ldg(c40 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
        cb[u] = t < q4 ? __ldg(c41 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const float4 a = xv[u];
        dot[0] = __fmaf_rn(a.x, ca[u].x, dot[0]);
        dot[0] = __fmaf_rn(a.y, ca[u].y, dot[0]);
        dot[0] = __fmaf_rn(a.z, ca[u].z, dot[0]);
        dot[0] = __fmaf_rn(a.w, ca[u].w, dot[0]);
        ab[0] = __fmaf_rn(fabsf(a.x), fabsf(ca[u].x), ab[0]);
        ab[0] = __fmaf_rn(fabsf(a.y), fabsf(ca[u].y), ab[0]);
        ab[0] = __fmaf_rn(fabsf(a.z), fabsf(ca[u].z), ab[0]);
        ab[0] = __fmaf_rn(fabsf(a.w), fabsf(ca[u].w), ab[0]);
        dot[1] = __fmaf_rn(a.x, cb[u].x, dot[1]);
        dot[1] = __fmaf_rn(a.y, cb[u].y, dot[1]);
        dot[1] = __fmaf_rn(a.z, cb[u].z, dot[1]);
        dot[1] = __fmaf_rn(a.w, cb[u].w, dot[1]);
        ab[1] = __fmaf_rn(fabsf(a.x), fabsf(cb[u].x), ab[1]);
        ab[1] = __fmaf_rn(fabsf(a.y), fabsf(cb[u].y), ab[1]);
        ab[1] = __fmaf_rn(fabsf(a.z), fabsf(cb[u].z), ab[1]);
        ab[1] = __fmaf_rn(fabsf(a.w), fabsf(cb[u].w), ab[1]);
      }
    } else {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        if (jc[h] == FALLBACK) continue;
        const float* cr = c + (long)jc[h] * d;
        for (int t = lane; t < d; t += 32) {
          const float xa = __ldg(xr + t), ca = __ldg(cr + t);
          dot[h] = __fmaf_rn(xa, ca, dot[h]);
          ab[h] = __fmaf_rn(fabsf(xa), fabsf(ca), ab[h]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      dot[0] = __fadd_rn(dot[0], __shfl_xor_sync(0xFFFFFFFFu, dot[0], o));
      ab[0] = __fadd_rn(ab[0], __shfl_xor_sync(0xFFFFFFFFu, ab[0], o));
      dot[1] = __fadd_rn(dot[1], __shfl_xor_sync(0xFFFFFFFFu, dot[1], o));
      ab[1] = __fadd_rn(ab[1], __shfl_xor_sync(0xFFFFFFFFu, ab[1], o));
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
      if (jc[h] == FALLBACK) break;
      float v, err;
      if (IP) {
        v = dot[h];
        err = __fmaf_ru(e2, ab[h], 1e-37f);
      } else {
        const float cj = __ldg(cn + jc[h]);
        v = __fsub_rn(cj, __fmul_rn(2.0f, dot[h]));
        // key error: twice the dot error plus the two key roundings.
        err = __fmaf_ru(2.0f * e2, ab[h], __fmaf_ru(ldexpf(1.0f, -22), fabsf(v), 1e-37f));
      }
      if (lane == 0) {
        pv[np] = v;
        pe[np] = err;
        pj[np] = jc[h];
      }
      np++;
    }
  }
  __syncwarp();
  // The best provable bound over the candidates, then every candidate that
  // could still beat it.
  float lim = IP ? -INFINITY : INFINITY;
  for (int e = lane; e < np; e += 32)
    lim = IP ? fmaxf(lim, __fsub_rd(pv[e], pe[e])) : fminf(lim, __fadd_ru(pv[e], pe[e]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ol = __shfl_xor_sync(0xFFFFFFFFu, lim, o);
    lim = IP ? fmaxf(lim, ol) : fminf(lim, ol);
  }
  int ns = 0;
  for (int base = 0; base < np; base += 32) {
    const int e = base + lane;
    const bool keep = e < np && (IP ? __fadd_ru(pv[e], pe[e]) >= lim
                                    : __fsub_rd(pv[e], pe[e]) <= lim);
    ns += __popc(__ballot_sync(0xFFFFFFFFu, keep));
  }
  // Each survivor becomes a (row, centroid) pair for the exact stage; the
  // row's result key starts at the identity of its reduction.
  const bool ok = ns >= 1 && ns <= SURV;
  uint32_t pbase = 0;
  if (lane == 0) {
    atomicAdd(&counters[2], (unsigned long long)np);
    if (ok) {
      pbase = atomicAdd(pair_count, (uint32_t)ns);
      rkey[i] = IP ? 0ull : ~0ull;
    } else {
      rkey[i] = IP ? 0ull : ~0ull;
      to_list((uint32_t)p, list, list_count, counters);
    }
  }
  pbase = __shfl_sync(0xFFFFFFFFu, pbase, 0);
  if (ok) {
    int w = 0;
    for (int base = 0; base < np; base += 32) {
      const int e = base + lane;
      const bool keep = e < np && (IP ? __fadd_ru(pv[e], pe[e]) >= lim
                                      : __fsub_rd(pv[e], pe[e]) <= lim);
      const uint32_t mask = __ballot_sync(0xFFFFFFFFu, keep);
      if (keep) pairs[pbase + w + __popc(mask & ((1u << lane) - 1u))] = make_uint2((uint32_t)i, pj[e]);
      w += __popc(mask);
    }
  }
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

// Exact chains over flattened (row, survivor) pairs, one thread per pair:
// x and the survivor's centroid stream through shared memory in 32-column
// slices (cp.async, 4 slices in flight), each 16-byte chunk q of pair slot t
// stored at q ^ (t & 7) so that the per-thread LDS.128 reads are free of bank
// conflicts. Each pair folds (value, id) into its row's 64-bit key with an
// atomic max (IP) / min (L2): the key orders by value, then by the lower id,
// which is the CPU's strict scan (-0.0 counts as +0.0, as it compares equal).
constexpr int EX_ROWS = 128, EX_COLS = 32, EX_STAGES = 4;

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

// Key of (v, j): larger key = better for IP (max v, then min j); smaller key
// = better for L2 (min v, then min j).
template <bool IP>
__device__ __forceinline__ unsigned long long result_key(float v, uint32_t j) {
  if (v == 0.0f) v = 0.0f;  // -0.0 == +0.0 in the CPU's comparisons
  const uint32_t u = __float_as_uint(v);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (IP ? (uint32_t)~j : j);
}

template <bool IP>
__global__ void __launch_bounds__(EX_ROWS) k_pairs(
    const float* __restrict__ x, int d, const uint32_t* __restrict__ ids, long p0,
    const float* __restrict__ c, const float* __restrict__ cn, const float* __restrict__ xnorm_row,
    const uint2* __restrict__ pairs, const uint32_t* __restrict__ pair_count,
    unsigned long long* __restrict__ rkey, float* __restrict__ xn_pos,
    uint32_t* __restrict__ bad) {
  extern __shared__ __align__(16) float ex_smem[];
  constexpr int SLICE = EX_STAGES * EX_ROWS * EX_COLS;
  float* xs = ex_smem;          // [stage][pair][32]
  float* cs = ex_smem + SLICE;  // [stage][pair][32]
  __shared__ const float* xrow_s[EX_ROWS];
  __shared__ const float* crow_s[EX_ROWS];
  const int t = threadIdx.x;
  const long np = (long)*pair_count;
  const int nsl = d / EX_COLS;
  const bool want_xn = !IP && !xnorm_row;
  for (long tile = blockIdx.x; tile * EX_ROWS < np; tile += gridDim.x) {
    const long pi = tile * EX_ROWS + t;
    const bool mine = pi < np;
    uint2 pr = make_uint2(0, 0);
    long row = 0;
    if (mine) {
      pr = pairs[pi];
      row = ids ? (long)ids[p0 + pr.x] : p0 + pr.x;
    }
    // Slots past the pair count read row 0 / centroid 0 harmlessly and write nothing.
    xrow_s[t] = x + row * (long)d;
    crow_s[t] = c + (long)pr.y * d;
    __syncthreads();
    auto issue = [&](int sl) {
      if (sl < nsl) {
        const int st = sl % EX_STAGES;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const int idx = u * EX_ROWS + t;  // 0 .. 1023
          const int r = idx >> 3, q = idx & 7;
          const int off = (st * EX_ROWS + r) * EX_COLS + (q ^ (r & 7)) * 4;
          const int g = sl * EX_COLS + q * 4;
          cp_async16(xs + off, xrow_s[r] + g);
          cp_async16(cs + off, crow_s[r] + g);
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
      __syncthreads();
      const int base = (sl % EX_STAGES * EX_ROWS + t) * EX_COLS;
      const float4* xr4 = reinterpret_cast<const float4*>(xs + base);
      const float4* cr4 = reinterpret_cast<const float4*>(cs + base);
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const int pq = q ^ (t & 7);
        const float4 a = xr4[pq], b = cr4[pq];
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
      __syncthreads();  // the slot is refilled next iteration
    }
    cp_async_wait<0>();
    if (mine) {
      const float v = IP ? acc : __fsub_rn(__ldg(cn + pr.y), __fmul_rn(2.0f, acc));
      if (!isfinite(v)) {
        bad[pr.x] = 1;  // overflowing chains: the exact scan reproduces the CPU here
      } else if (IP) {
        atomicMax(rkey + pr.x, result_key<IP>(v, pr.y));
      } else {
        atomicMin(rkey + pr.x, result_key<IP>(v, pr.y));
      }
      if (want_xn) xn_pos[pr.x] = xn;  // the same value from every pair of the row
    }
    __syncthreads();  // row pointers are rewritten by the next tile
  }
}

// The same for d % 32 != 0: one thread per pair reads its operands directly.
template <bool IP>
__global__ void k_pairs_plain(const float* __restrict__ x, int d, const uint32_t* __restrict__ ids,
                              long p0, const float* __restrict__ c, const float* __restrict__ cn,
                              const float* __restrict__ xnorm_row, const uint2* __restrict__ pairs,
                              const uint32_t* __restrict__ pair_count,
                              unsigned long long* __restrict__ rkey, float* __restrict__ xn_pos,
                              uint32_t* __restrict__ bad) {
  const long np = (long)*pair_count;
  for (long pi = (long)blockIdx.x * blockDim.x + threadIdx.x; pi < np;
       pi += (long)gridDim.x * blockDim.x) {
    const uint2 pr = pairs[pi];
    const long row = ids ? (long)ids[p0 + pr.x] : p0 + pr.x;
    const float* xr = x + row * (long)d;
    const float acc = chain(xr, c + (long)pr.y * d, d);
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

// Labels and scores from the rows' keys; rows whose chains overflowed join
// the exact kernel's list.
template <bool IP>
__global__ void k_finish(const uint32_t* __restrict__ ids, long p0, long m,
                         const float* __restrict__ xnorm_row, const float* __restrict__ xn_pos,
                         const unsigned long long* __restrict__ rkey, uint32_t* __restrict__ bad,
                         uint32_t* __restrict__ labels, float* __restrict__ scores,
                         uint32_t* __restrict__ list, uint32_t* __restrict__ list_count,
                         unsigned long long* __restrict__ counters) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const unsigned long long key = rkey[i];
  if (bad[i]) {
    bad[i] = 0;
    to_list((uint32_t)(p0 + i), list, list_count, counters);
    return;
  }
  if (key == (IP ? 0ull : ~0ull)) return;  // on the list already (or no pair)
  const uint32_t ord = (uint32_t)(key >> 32);
  const uint32_t u = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
  const float v = __uint_as_float(u);
  const uint32_t j = IP ? ~(uint32_t)key : (uint32_t)key;
  float score = v;
  if (!IP) {
    const long row = ids ? (long)ids[p0 + i] : p0 + i;
    score = fmaxf(__fadd_rn(xnorm_row ? xnorm_row[row] : xn_pos[i], v), 0.0f);
  }
  labels[p0 + i] = j;
  scores[p0 + i] = score;
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

// A 2-D FP16 tensor map over rows x dp (row stride dp*2 bytes) with a
// box of `box_rows` x 64 columns and 128-byte swizzle.
CUtensorMap make_map(const void* base, size_t rows, size_t dp, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)dp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)dp * 2};
  cuuint32_t box[2] = {(cuuint32_t)BKH, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(EB_ERROR, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

// The dynamic shared memory limit is a per-device, per-kernel attribute.
template <bool IP>
void set_smem(int device) {
  static uint64_t done = 0;  // one instance per kernel: IP is a template parameter
  if (!(done >> device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_screen<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SMEM_BYTES));
    done |= 1ull << device;
  }
}

template <bool IP>
void set_exact_smem(int device, size_t bytes) {
  static uint64_t done = 0;
  if (!(done >> device & 1)) {
    EB_CUDA(cudaFuncSetAttribute(k_pairs<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)bytes));
    done |= 1ull << device;
  }
}

}  // namespace

bool top1_screen_supported(eb_engine* e, const Top1Args& a) {
  if (e->screen_mode == 0) return false;
  if (a.d > 16384 || a.k > 0x7FFFFFFF) return false;
  if (e->screen_mode == 2) return true;
  return a.k >= 64 && a.r1 - a.r0 >= 128 && a.d >= 16;
}

void top1_screen(eb_engine* e, const Top1Args& a, eb_buf* xbuf) {
  const size_t d = a.d, k = a.k;
  const size_t dp = (d + BKH - 1) / BKH * BKH;
  const size_t m_all = a.r1 - a.r0;
  // Rows per pass: eight 128-row tiles per SM, so that each persistent CTA
  // keeps its operand ring and TMEM buffers running across tiles.
  const size_t wave = (size_t)e->num_sms * BM;
  const size_t chunk = std::min(m_all, PASS_WAVES * wave);
  const bool ip = a.metric == EB_IP;

  // Bound coefficients for this d (see the header comment), with 1% slack.
  const double dd = (double)d;
  const double gamma_d = dd * std::ldexp(1.0, -24) / (1.0 - dd * std::ldexp(1.0, -24));
  const float e_rel = (float)((std::ldexp(1.0, -10) + std::ldexp(1.0, -22) +
                               dd * std::ldexp(1.0, -21) * (1.0 + std::ldexp(1.0, -9)) + gamma_d) *
                              1.01);
  const float e_abs = (float)(std::ldexp(1.0, -24) * std::sqrt(dd) * 1.01);
  const float e_min = (float)(dd * std::ldexp(1.0, -50));

  // Centroids: one exponent, FP16 copy.
  uint32_t* cinfo = e->scratch_get<uint32_t>("tc_cinfo", 4);
  __half* ch = e->scratch_get<__half>("tc_ch", k * dp);
  EB_CUDA(cudaMemsetAsync(cinfo, 0, 16, e->stream));
  const unsigned wpb = 8;
  k_cent_max<<<(unsigned)((k + wpb - 1) / wpb), wpb * 32, 0, e->stream>>>(a.c, (long)k, (int)d,
                                                                          cinfo);
  EB_LAUNCH("screen centroid max");
  k_cent_conv<<<(unsigned)((k + wpb - 1) / wpb), wpb * 32, 0, e->stream>>>(
      a.c, (long)k, (int)d, (int)dp, cinfo, ch);
  EB_LAUNCH("screen centroid convert");
  const CUtensorMap mapB = make_map(ch, k, dp, BN);

  __half* xh = e->scratch_get<__half>("tc_xh", chunk * dp);
  int* xexp = e->scratch_get<int>("tc_xexp", chunk);
  float* xnrm = e->scratch_get<float>("tc_xnrm", chunk);
  uint2* cand = e->scratch_get<uint2>("tc_cand", chunk * CAP);
  uint32_t* cand_cnt = e->scratch_get<uint32_t>("tc_cnt", chunk);
  float* cand_thr = e->scratch_get<float>("tc_thr", chunk);
  uint2* pairs = e->scratch_get<uint2>("tc_pairs", chunk * SURV);
  uint32_t* pair_count = e->scratch_get<uint32_t>("tc_pair_count", 4);
  unsigned long long* rkey = e->scratch_get<unsigned long long>("tc_rkey", chunk);
  uint32_t* bad = e->scratch_get<uint32_t>("tc_bad", chunk);
  float* xn_pos = e->scratch_get<float>("tc_xn_pos", chunk);
  // Precise-dot bound of the refine stage: each lane's FMA chain plus the
  // 5-level shuffle tree is at most kp roundings, gamma_kp sum|x c|; the exact
  // chain adds gamma_d sum|x c|; the computed sum|x c| is itself within gamma_kp.
  const double kp = std::ceil(dd / 32.0) + 5.0;
  const double gamma_kp = kp * std::ldexp(1.0, -24) / (1.0 - kp * std::ldexp(1.0, -24));
  const float e2 = (float)((gamma_kp + gamma_d) * (1.0 + 4.0 * gamma_kp) * 1.01);
  uint32_t* list = e->scratch_get<uint32_t>("tc_list", chunk);
  uint32_t* list_count = e->scratch_get<uint32_t>("tc_list_count", 4);
  unsigned long long* counters = e->counters();

  ScreenParams P;
  P.k = (int)k;
  P.kblocks = (int)(dp / BKH);
  P.ntiles = (int)((k + BN - 1) / BN);
  P.d = (int)d;
  P.xexp = xexp;
  P.xnrm = xnrm;
  P.cn = a.cnorm;
  P.cinfo = cinfo;
  P.e_rel = e_rel;
  P.e_abs = e_abs;
  P.e_min = e_min;
  P.cand = cand;
  P.cand_cnt = cand_cnt;
  P.cand_thr = cand_thr;
  P.status = e->d_status;

  if (ip)
    set_smem<true>(e->device);
  else
    set_smem<false>(e->device);

  // A bound data set keeps its FP16 screen copy across calls (training steps,
  // repeated assigns): converted once, then read in place or gathered by id.
  Fp16Copy* cache = nullptr;
  if (xbuf && xbuf->d == d && xbuf->len == a.n * d) {
    if (xbuf->f16 && xbuf->f16->version != xbuf->version) drop_f16(xbuf);
    if (!xbuf->f16) {
      auto* f = new Fp16Copy;
      f->n = a.n;
      f->d = d;
      f->version = xbuf->version;
      f->stream = e->stream;
      cudaError_t st = cudaMallocAsync(&f->xh, std::max<size_t>(a.n * dp, 8) * 2, e->stream);
      if (st == cudaSuccess) st = cudaMallocAsync(&f->xexp, std::max<size_t>(a.n, 1) * 4, e->stream);
      if (st == cudaSuccess) st = cudaMallocAsync(&f->xnrm, std::max<size_t>(a.n, 1) * 4, e->stream);
      xbuf->f16 = f;
      if (st != cudaSuccess) {
        drop_f16(xbuf);  // no room for the copy: convert per pass instead
        cudaGetLastError();
      } else if (a.n) {
        k_prep_rows<<<(unsigned)((a.n + wpb - 1) / wpb), wpb * 32, 0, e->stream>>>(
            a.x, (long)a.n, (int)d, (int)dp, nullptr, 0, (long)a.n, f->xh, f->xexp, f->xnrm,
            e->d_status);
        EB_LAUNCH("screen copy of bound rows");
      }
    }
    cache = xbuf->f16;
  }

  for (size_t c0 = a.r0; c0 < a.r1; c0 += chunk) {
    const size_t m = std::min(chunk, a.r1 - c0);
    const __half* xa = xh;
    if (cache && !a.ids) {
      // Dense rows of the bound set: the screen reads the cached copy in place.
      xa = cache->xh + c0 * dp;
      P.xexp = cache->xexp + c0;
      P.xnrm = cache->xnrm + c0;
    } else if (cache) {
      k_gather_rows<<<(unsigned)((m + wpb - 1) / wpb), wpb * 32, 0, e->stream>>>(
          cache->xh, cache->xexp, cache->xnrm, (long)a.n, (int)dp, a.ids, (long)c0, (long)m, xh,
          xexp, xnrm, e->d_status);
      EB_LAUNCH("screen row gather");
      P.xexp = xexp;
      P.xnrm = xnrm;
    } else {
      k_prep_rows<<<(unsigned)((m + wpb - 1) / wpb), wpb * 32, 0, e->stream>>>(
          a.x, (long)a.n, (int)d, (int)dp, a.ids, (long)c0, (long)m, xh, xexp, xnrm, e->d_status);
      EB_LAUNCH("screen row prep");
      P.xexp = xexp;
      P.xnrm = xnrm;
    }
    const CUtensorMap mapA = make_map(xa, m, dp, BM);
    P.m = (long)m;
    // Persistent: at most one CTA per SM, each looping over row tiles.
    const unsigned grid = (unsigned)std::min<size_t>((m + BM - 1) / BM, (size_t)e->num_sms);
    if (ip)
      k_screen<true><<<grid, NTHREADS, SMEM_BYTES, e->stream>>>(mapA, mapB, P);
    else
      k_screen<false><<<grid, NTHREADS, SMEM_BYTES, e->stream>>>(mapA, mapB, P);
    EB_LAUNCH("screen");
    EB_CUDA(cudaMemsetAsync(list_count, 0, 4, e->stream));
    EB_CUDA(cudaMemsetAsync(pair_count, 0, 4, e->stream));
    EB_CUDA(cudaMemsetAsync(bad, 0, m * sizeof(uint32_t), e->stream));
    const unsigned rgrid = (unsigned)((m + 7) / 8);  // 8 rows (warps) per block
    if (ip)
      k_refine<true><<<rgrid, 256, 0, e->stream>>>(a.x, (int)d, a.ids, (long)c0, (long)m, a.c,
                                                   a.cnorm, cand, cand_cnt, cand_thr, e2, pairs,
                                                   pair_count, rkey, list, list_count, counters);
    else
      k_refine<false><<<rgrid, 256, 0, e->stream>>>(a.x, (int)d, a.ids, (long)c0, (long)m, a.c,
                                                    a.cnorm, cand, cand_cnt, cand_thr, e2, pairs,
                                                    pair_count, rkey, list, list_count, counters);
    EB_LAUNCH("screen refine");
    // The pair count is known on the device only: persistent blocks stride over it.
    const unsigned pgrid = (unsigned)e->num_sms;
    if (d % EX_COLS == 0) {
      const size_t ex_smem = 2 * EX_STAGES * EX_ROWS * EX_COLS * sizeof(float);
      if (ip) {
        set_exact_smem<true>(e->device, ex_smem);
        k_pairs<true><<<pgrid, EX_ROWS, ex_smem, e->stream>>>(a.x, (int)d, a.ids, (long)c0, a.c,
                                                              a.cnorm, a.xnorm, pairs, pair_count,
                                                              rkey, xn_pos, bad);
      } else {
        set_exact_smem<false>(e->device, ex_smem);
        k_pairs<false><<<pgrid, EX_ROWS, ex_smem, e->stream>>>(a.x, (int)d, a.ids, (long)c0, a.c,
                                                               a.cnorm, a.xnorm, pairs, pair_count,
                                                               rkey, xn_pos, bad);
      }
    } else {
      if (ip)
        k_pairs_plain<true><<<pgrid * 4, 128, 0, e->stream>>>(a.x, (int)d, a.ids, (long)c0, a.c,
                                                              a.cnorm, a.xnorm, pairs, pair_count,
                                                              rkey, xn_pos, bad);
      else
        k_pairs_plain<false><<<pgrid * 4, 128, 0, e->stream>>>(a.x, (int)d, a.ids, (long)c0, a.c,
                                                               a.cnorm, a.xnorm, pairs,
                                                               pair_count, rkey, xn_pos, bad);
    }
    EB_LAUNCH("screen exact chains");
    const unsigned fgrid = (unsigned)((m + 255) / 256);
    if (ip)
      k_finish<true><<<fgrid, 256, 0, e->stream>>>(a.ids, (long)c0, (long)m, a.xnorm, xn_pos, rkey,
                                                   bad, a.labels, a.scores, list, list_count,
                                                   counters);
    else
      k_finish<false><<<fgrid, 256, 0, e->stream>>>(a.ids, (long)c0, (long)m, a.xnorm, xn_pos,
                                                    rkey, bad, a.labels, a.scores, list,
                                                    list_count, counters);
    EB_LAUNCH("screen finish");
    Top1Args fa = a;
    fa.r0 = c0;
    fa.r1 = c0 + m;
    top1_exact_list(e, fa, list, list_count, m);
  }
  e->stats.screened_rows += m_all;
}

}  // namespace eb
