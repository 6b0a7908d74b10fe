// Internal declarations shared by the engine's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdio>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/emeans_b200.h"

namespace eb {

// An error that becomes a status code at the C ABI edge.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void ensure(bool ok, const std::string& msg) {
  if (!ok) throw Error(EB_INVALID_ARGUMENT, msg);
}
// A literal message builds no string unless the check fails (checks run in
// per-element loops).
inline void ensure(bool ok, const char* msg) {
  if (!ok) throw Error(EB_INVALID_ARGUMENT, msg);
}

inline void cuda_check(cudaError_t st, const char* what) {
  if (st != cudaSuccess)
    throw Error(EB_ERROR, std::string(what) + ": " + cudaGetErrorString(st));
}
#define EB_CUDA(x) ::eb::cuda_check((x), #x)
// After every kernel launch: check the launch and count it (eb_stats).
#define EB_LAUNCH(what)                              \
  do {                                               \
    ::eb::cuda_check(cudaGetLastError(), what);      \
    e->stats.kernel_launches++;                      \
  } while (0)

// Device-side error flags (a word in device memory; read by the next sync).
enum : uint32_t {
  ST_BAD_LABEL = 1u,
  ST_BAD_ROW = 2u,
  ST_WAIT_TIMEOUT = 4u,
  ST_BAD_STATE = 8u,  // a kernel found an index its producer should never write
};

// A grow-only device scratch slot.
struct Scratch {
  void* p = nullptr;
  size_t bytes = 0;
};

struct Fp16Copy;  // split FP16 screen copy of a bound data set (top1_tc.cu)
struct PeerExchange;  // a group's symmetric exchange region (nccl.cpp)
// Words of flags before the data of an exchange region (ready [0, 64), done
// [64, 128), a block ticket at 128; 1 KB, so the data is 16-byte aligned).
constexpr size_t kPxFlagWords = 256;
struct Q8Copy;    // fixed-point screen copy of a bound data set (top1_tc.cu)

}  // namespace eb

struct eb_buf {
  void* ptr = nullptr;
  size_t len = 0;
  int dtype = EB_F32;
  bool owned = false;
  // Bumped by every host write; caches derived from the buffer compare it.
  uint64_t version = 0;
  // For bound data sets: d, the rows' squared norms (CPU float order) and the
  // screen copies (split FP16 for the internal scores' products, fixed point
  // for top-1).
  size_t d = 0;
  float* xnorm = nullptr;
  eb::Fp16Copy* f16 = nullptr;
  eb::Q8Copy* q8 = nullptr;
};

struct eb_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t* d_status = nullptr;  // device error flags
  uint32_t* h_status = nullptr;  // pinned mirror
  std::unordered_map<std::string, eb::Scratch> scratch;
  eb_stats stats{};
  // Assigner::bind_data state.
  eb_buf* bound = nullptr;
  const float* bound_host = nullptr;
  size_t bound_n = 0;
  int num_sms = 148;
  // Device allocations the engine has made since creation (buffers, scratch,
  // cached copies), for callers that check a call allocated nothing.
  uint64_t device_allocs = 0;
  // Failure-detection test: the next top-1 screen launch makes one wait run
  // out (eb_test_screen_dead_wait); cleared by that launch.
  int screen_dead_wait = 0;
  // Tensor-core screen for top-1: 0 off, 1 auto (large enough calls), 2 always.
  // EMEANS_B200_SCREEN=0/1/2 sets it at creation; eb_set_screen_mode later.
  int screen_mode = 1;
  // Device counters: [0] unused, [1] fallback rows, [2] re-scored candidates.
  unsigned long long* d_counters = nullptr;
  // Multi-GPU group (eb_engine_join): an NCCL communicator over one engine per
  // GPU, or null for a single-GPU engine.
  void* comm = nullptr;
  int rank = 0, world = 1;
  // Group training: 0 splits a batch's top-1 across the ranks only when that
  // shortens it, 1 always, 2 never, 3 splits the top-1 and the scatter-add
  // and sums the ranks' partial sums (eb_set_group_shard).
  int group_shard = 0;
  // The group's symmetric exchange region (eb_group_exchange), or null, and
  // why the last set-up did not map one.
  eb::PeerExchange* px = nullptr;
  std::string px_why;
  // Optional CUDA-event timing of the top-1 screen kernel (eb_set_kernel_timing):
  // one (start, end) pair per launch since the last eb_screen_timing read,
  // with the rows of that launch.
  // Second stream for host-to-device copies that overlap compute (eb_assign,
  // training's epoch orders) and a third for training's epoch read-backs,
  // created on first use.
  cudaStream_t copy_stream = nullptr;
  cudaStream_t down_stream = nullptr;
  bool time_screen = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> screen_ev;
  std::vector<size_t> screen_ev_rows;
  size_t screen_ev_used = 0;
  // Generation of the screen's centroid summary (max |c|, norm bound,
  // non-finite flag): each conversion of a centroid set tags its atomics with
  // a new generation, so the summary needs no zeroing pass per call.
  uint32_t cinfo_gen = 0;
  unsigned long long* counters() { return d_counters; }
  // Events of the two pinned staging buffers of caller copies (hostcopy.cpp).
  cudaEvent_t stage_ev[2] = {nullptr, nullptr};
  // Pinned host buffers (training read-backs, staging), grown on demand,
  // freed with the engine.
  std::unordered_map<std::string, eb::Scratch> pinned;
  template <class T>
  T* pinned_get(const char* name, size_t count) {
    auto& s = pinned[name];
    size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    if (s.bytes < bytes) {
      if (s.p) {
        EB_CUDA(cudaStreamSynchronize(stream));  // no copy may still target it
        cudaFreeHost(s.p);
        s.p = nullptr;
        s.bytes = 0;
      }
      EB_CUDA(cudaMallocHost(&s.p, bytes));
      s.bytes = bytes;
    }
    return static_cast<T*>(s.p);
  }

  // Scratch that grows on demand; with `zeroed`, a new allocation is zeroed
  // (on the stream) before first use.
  template <class T>
  T* scratch_get(const char* name, size_t count, bool zeroed = false) {
    auto& s = scratch[name];
    size_t bytes = count * sizeof(T);
    if (bytes == 0) bytes = 16;
    if (s.bytes < bytes) {
      if (s.p) EB_CUDA(cudaFreeAsync(s.p, stream));
      size_t want = bytes + bytes / 4;
      EB_CUDA(cudaMallocAsync(&s.p, want, stream));
      device_allocs++;
      s.bytes = want;
      if (zeroed) EB_CUDA(cudaMemsetAsync(s.p, 0, want, stream));
    }
    return static_cast<T*>(s.p);
  }
};

namespace eb {

#ifndef EB_PDL
#define EB_PDL 1
#endif
#ifdef __CUDACC__
// Programmatic dependent launch: kernels on the hot paths are launched with
// launch_pdl, which lets the device schedule a kernel while its predecessor on
// the stream drains (no launch gap); every such kernel begins with pdl_wait(),
// which returns once the predecessor has completed and its writes are
// visible. In a kernel launched without the attribute it returns at once.
// (Measured: also letting the next kernel be scheduled as soon as every
// block of this one has started, griddepcontrol.launch_dependents, made the
// training loop slower.)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// A word of the screen's centroid summary (generation << 32 | payload, only
// ever raised) raised to at least v. Most contributions do not raise it: the
// word is read first (from L2) and only a larger v goes to the atomic, so
// that a thousand blocks do not queue on one address.
__device__ __forceinline__ void summary_max(unsigned long long* w, unsigned long long v) {
  if (__ldcg(w) < v) atomicMax(w, v);
}

template <typename... KArgs, typename... Args>
void launch_pdl(eb_engine* e, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = EB_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cuda_check(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), "kernel launch");
}
#endif

eb_buf* new_buf(eb_engine* e, int dtype, size_t len);
// Copies of caller host memory (hostcopy.cpp): pinned memory directly,
// pageable memory through the engine's pinned staging buffers. h2d returns
// once the source may be reused (the last DMA may still be in flight on st);
// d2h returns once dst holds the data.
bool host_pinned(const void* p);
void h2d(eb_engine* e, void* dst, const void* src, size_t bytes, cudaStream_t st);
void d2h(eb_engine* e, void* dst, const void* src, size_t bytes, cudaStream_t st);
void free_buf(eb_engine* e, eb_buf* b);
void sync(eb_engine* e);  // wait + status check (throws)
void set_last_error(const std::string& msg);

// Group exchange (nccl.cpp): in-place all-gather of `words` 32-bit words per
// rank in buf[0 .. world * words) on the engine's stream; rank r's share is
// buf[r * words ..). Release of the engine's communicator.
void group_allgather(eb_engine* e, uint32_t* buf, size_t words);
void group_leave(eb_engine* e);
// ops.cu: the all-gather over the group's exchange regions (peers_d: every
// rank's region on this GPU, own included); words per rank, a multiple of 4.
void px_allgather(eb_engine* e, uint32_t* const* peers_d, int world, int rank, size_t words,
                  uint32_t epoch);
// Pack this rank's (labels, scores) slice of len <= soff entries into
// stage[rank * stride ..) (labels, then scores soff words later; the words
// past len zero) and unpack every rank's slice after the exchange into
// labels / scores at p0 + q s, rank q's slice being positions q s .. (q + 1) s
// of the batch (ops.cu). stride >= 2 soff words separates the ranks' shares.
void shard_pack(eb_engine* e, const uint32_t* labels, const float* scores, size_t len,
                size_t soff, size_t stride, uint32_t* stage);
void shard_unpack(eb_engine* e, const uint32_t* stage, size_t total, size_t s, size_t soff,
                  size_t stride, uint32_t* labels, float* scores);
// The group's partial scatter-adds summed in rank order: every rank's share of
// stage (stride words apart) holds its counts (k words at cnt_off) and sums
// (k x d floats at sum_off); sums = ((p_0 + p_1) + p_2) + ..., counts = the
// total, and acc += sums when acc is given (ops.cu).
void reduce_partials(eb_engine* e, const uint32_t* stage, size_t stride, int world,
                     size_t cnt_off, size_t sum_off, size_t k, size_t d, float* sums,
                     uint32_t* counts, float* acc);

// ---- ops.cu: update ops, bit-equal to the CPU float order
void row_norms(eb_engine* e, const float* m, size_t rows, size_t d, float* out);
// Squared norms of the selected rows x[ids[p]] (or x[p]) for p in r0..r1,
// written at out[p - r0].
void sel_row_norms(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* ids,
                   size_t r0, size_t r1, float* out);
void normalize_rows(eb_engine* e, const float* src, size_t rows, size_t d, float* dst);
void ema_update(eb_engine* e, float* pos, float* usage, const float* sums, const uint32_t* counts,
                size_t k, size_t d, float alpha, float decay, bool replace);
void split(eb_engine* e, float* pos, float* usage, const uint32_t* d_pairs, size_t npairs,
           size_t d);
// ema_update followed by the next step's readout of the updated centroids
// (L2: their squared norms into readout[k]; spherical: their normalised rows
// into readout[k x d]) and the screen's summary of the centroids the next
// top-1 reads (generation gen of the engine's summary words cinfo), in one
// kernel; results bit-equal to ema_update + row_norms / normalize_rows. False
// (nothing launched) when d is too large for the kernel's shared memory.
bool ema_update_readout(eb_engine* e, float* pos, float* usage, const float* sums,
                        const uint32_t* counts, size_t k, size_t d, float alpha, float decay,
                        bool replace, bool spherical, float* readout,
                        unsigned long long* cinfo, uint32_t gen);
// The screen's centroid summary words and a fresh generation for them
// (top1_tc.cu); a Top1Args with summary_gen set to it skips the summary pass.
unsigned long long* screen_summary_words(eb_engine* e);
uint32_t screen_next_summary_gen(eb_engine* e);
void scatter_add(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0,
                 size_t r1, const uint32_t* labels, size_t k, float* sums, uint32_t* counts,
                 float* acc);
// Stable counting sort of the selected positions r0..r1 by label: counts[l]
// (device), start[0..k] (exclusive prefix, engine scratch) and order[start[l]
// ..] = the data rows of label l in selection order (engine scratch); with
// by_size, the labels by count, largest first (engine scratch).
void label_order(eb_engine* e, const uint32_t* ids, size_t r0, size_t r1, size_t n,
                 const uint32_t* labels, size_t k, uint32_t* counts, const uint32_t** order,
                 const uint32_t** start, const uint32_t** by_size = nullptr);
// ---- metrics.cu: internal quality scores of a labelling
void internal_scores(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* labels,
                     size_t k, eb_internal* out, uint64_t* sizes);
// cnt[l] = occurrences of label l in labels[0 .. m).
void label_counts(eb_engine* e, const uint32_t* labels, size_t m, size_t k, uint32_t* cnt);
// out = sums / count per centroid, pos where the count is 0 (closing means
// before any renormalisation).
void closing_means(eb_engine* e, const float* pos, const float* sums, const uint32_t* cnt,
                   size_t k, size_t d, float* out);

// ---- top1_exact.cu: the exact FP32 SIMT kernels
struct Top1Args {
  const float* x;      // n x d
  size_t n, d;
  const uint32_t* ids; // selection ids or null
  size_t r0, r1;       // positions
  const float* c;      // k x d
  const float* cnorm;  // k (L2)
  size_t k;
  int metric;
  uint32_t* labels;    // indexed by position
  float* scores;
  const float* xnorm;  // squared norms by data row (L2), or null: computed
  // The tensor-core screen's split copy of these centroids is already in its
  // scratch (a later slice of the same call): skip the conversion.
  bool centroids_ready = false;
  // Nonzero: the screen's summary of these centroids (max |c|, norm bound,
  // non-finite flag) is already in the engine's summary words under this
  // generation (written by ema_update_readout): only the split copy is made.
  uint32_t summary_gen = 0;
};
// Full exact scan of every selected row.
void top1_exact(eb_engine* e, const Top1Args& a);

// Screen when the tensor-core path supports the call, else the exact kernel.
void top1_dispatch(eb_engine* e, const Top1Args& a, eb_buf* xbuf);

// ---- top1_tc.cu: the tcgen05 screen + exact re-score
// Parts per row tile of a screen pass over rtiles row tiles, and the screen's
// estimated length in centroid-tile times for `rows` rows against k centroids.
int screen_parts(size_t rtiles, int ntiles, int sms);
// The internal scores' product on the tensor cores (top1_tc.cu):
// best_out[i] = the centroid s other than slot[labels[i]] with the largest
// x_i . c_s * inv[s] (split FP16 products with FP32 accumulation);
// 0xFFFFFFFF when there is none, 0xFFFFFFFE when the row could not be scored.
void screen_products(eb_engine* e, const float* x, size_t n, size_t d, eb_buf* xbuf,
                     const uint32_t* labels, const uint32_t* slot, const float* c,
                     const float* inv, size_t k, uint32_t* best_out);
size_t screen_tile_times(size_t rows, size_t k, int sms);
bool top1_screen_supported(eb_engine* e, const Top1Args& a);
void top1_screen(eb_engine* e, const Top1Args& a, eb_buf* xbuf);
void drop_f16(eb_buf* b);  // drops both screen copies
// The bound set's split copy (made on first use; null if xbuf is not a bound
// set of that shape or there is no room).
Fp16Copy* bound_copy(eb_engine* e, eb_buf* xbuf, const float* x, size_t n, size_t d);

// ---- topk.cu
void topk(eb_engine* e, const float* q, size_t m, const float* data, size_t n, size_t d,
          size_t kk, bool exclude_self, uint32_t* ids, float* sims, size_t id0 = 0,
          bool collective = false);
// Exact top-kk of L device-resident queries against n device-resident data
// rows, results on the device (topk.cu).
void topk_exact_device(eb_engine* e, const float* q, size_t L, const uint32_t* qids,
                       const float* data, size_t n, size_t d, size_t kk, bool exclude_self,
                       uint32_t* ids, float* sims, size_t id0);
// Top-kk on the tensor-core screen (top1_tc.cu): queries and data on the
// device, data row j with global id id0 + j; results (global ids) on the
// device. False when the call is not one it takes.
bool topk_screen(eb_engine* e, const float* q, size_t m, const float* data, size_t n, size_t d,
                 size_t kk, bool exclude_self, uint32_t* ids, float* sims, size_t id0);

}  // namespace eb
