/*
 * emeans_b200: a B200 (sm_100a) engine for the emeans hot path, behind a C ABI.
 *
 * The ABI mirrors the reference's layer-1 op contract, `trait Device`
 * (crates/emeans-core/src/core/mod.rs:71-178), one entry point per method, so
 * that a thin Rust crate can implement `Device + Assigner` over it and plug in
 * at `make_assigner(Backend::Cuda)` (crates/emeans-cluster/src/backend.rs:126-133).
 * Above it, `eb_assign` is `Assigner::assign` (crates/emeans-core/src/assign.rs:71-117,
 * core::assign_on core/mod.rs:249-330) and `eb_train` is `Engine::run_train`
 * (core/mod.rs:229-231), the reference device loop (core/train.rs:60-303)
 * restated in C++ on this engine.
 *
 * Conventions (from crates/emeans-ffi/include/emeans.h:66-80 and
 * crates/emeans-ffi/src/lib.rs:95-126):
 *  - every function returns a status code; on failure eb_last_error() holds a
 *    message for the calling thread;
 *  - ops are queued on the engine's stream and only eb_buf_read / eb_sync (and
 *    the host-array entry points eb_assign, eb_topk, eb_train) wait; errors
 *    that a kernel detects (a label >= k, a row id past the data) are
 *    reported by the next call that waits, as EB_INVALID_ARGUMENT;
 *  - an engine is owned by one thread at a time (Send, not Sync);
 *  - outputs outside the selection rows r0..r1 are never written.
 *
 * Exactness (the reference contract, core/mod.rs:60-69):
 *  - eb_top1 / eb_assign: labels and scores bit-equal to the reference CPU
 *    kernel (`cpu-fused`, assign/fused.rs): each dot is one sequential FMA
 *    chain over d; ties keep the lower id; L2 keys are cnorm - 2 dot (one
 *    rounding) and scores max(sum x^2 + key, 0). The tensor-core screen only
 *    chooses which centroids get the exact FP32 chain.
 *  - eb_scatter_add: counts exact; sums bit-equal to adding the rows in
 *    selection order in f32.
 *  - eb_ema_update, eb_split, eb_row_norms, eb_normalize_rows: bit-equal to
 *    the CPU float order (no FMA contraction, IEEE divide and sqrt).
 *  - eb_topk: ids and scores bit-equal to the exact top-k by FMA-chain inner
 *    product (best first, lower id on ties).
 */
#ifndef EMEANS_B200_H
#define EMEANS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: crates/emeans-ffi/include/emeans.h:66-80. */
#define EB_OK 0
#define EB_INVALID_ARGUMENT 1
#define EB_ERROR 2 /* CUDA/NCCL failure, out of memory, device-wait timeout */
#define EB_INTERNAL 3

/* Element types of engine buffers. */
#define EB_F32 0
#define EB_U32 1

/* Metric: crates/emeans-core/src/assign.rs:14-21. */
#define EB_L2 0
#define EB_IP 1

typedef struct eb_engine eb_engine;
typedef struct eb_buf eb_buf;

/* Message of the last failed call on this thread ("" if none). */
const char* eb_last_error(void);
/* Library version string. */
const char* eb_version(void);

/* ---------------------------------------------------------------- engine */

/* An engine on CUDA device `device` with its own stream. No device, or a
 * device that is not sm_100, fails with EB_ERROR
 * (crates/emeans-cuda/src/lib.rs:303-309: a missing driver is an error). */
int eb_engine_create(int device, eb_engine** out);
int eb_engine_destroy(eb_engine* e);
/* Device::name (core/mod.rs:77). Writes a NUL-terminated name. */
int eb_engine_name(eb_engine* e, char* buf, size_t cap);
/* Device::flush (core/mod.rs:93-95): submit queued work without waiting. */
int eb_flush(eb_engine* e);
/* Wait for queued work; report errors detected on the device. */
int eb_sync(eb_engine* e);

/* The engine's CUDA stream (a cudaStream_t), for callers that order their own
 * work or CUDA events against the engine's. */
int eb_engine_stream(eb_engine* e, void** stream);

/* Counters since creation: rows top-1 screened on tensor cores, rows that fell
 * back to the exact full scan, candidates re-scored exactly, rows served by the
 * exact SIMT kernel directly, kernels launched, and bytes of caller memory
 * copied to the device by the buffer, bind, assign, top-k and internal-scores
 * calls (rows, centroids, labels; not the training loop's own small
 * uploads). */
typedef struct {
  uint64_t screened_rows;
  uint64_t fallback_rows;
  uint64_t rescored_candidates;
  uint64_t exact_rows;
  uint64_t kernel_launches;
  uint64_t h2d_bytes;
} eb_stats;
int eb_get_stats(eb_engine* e, eb_stats* out);

/* No counterpart in the reference: a failure-detection test hook. With on,
 * the next launch of the top-1 tensor-core screen has its first CTA's
 * epilogue wait, at its second centroid tile, on a device barrier that
 * nothing arrives at; the wait gives up after its limit (2 s), the CTA's
 * other roles see the abort, wait for their own copies and products in flight
 * and free their tensor memory, its rows go to the exact full scan, and the
 * next synchronising call reports EB_ERROR ("device-side wait timed out").
 * The labels and scores are still exact; the engine stays usable. The hook
 * clears itself at that launch. */
int eb_test_screen_dead_wait(eb_engine* e, int on);

/* No counterpart in the reference. The number of device allocations the
 * engine has made since creation (buffers, grow-only scratch, cached copies of
 * bound data); a call that allocated nothing leaves it unchanged. */
int eb_device_allocations(eb_engine* e, uint64_t* count);

/* Top-1 path: 0 = exact SIMT kernel only, 1 = tensor-core screen + exact
 * re-score for calls large enough to pay (the default), 2 = screen always.
 * Results are identical in every mode; only the speed differs. The
 * environment variable EMEANS_B200_SCREEN=0/1/2 sets it at engine creation. */
int eb_set_screen_mode(eb_engine* e, int mode);

/* No counterpart in the reference (measurement only). With timing on, every
 * launch of the top-1 tensor-core screen kernel is bracketed by CUDA events on
 * the engine's stream; eb_screen_timing waits for queued work and returns the
 * launches since the last read, their summed device time and their rows. */
int eb_set_kernel_timing(eb_engine* e, int on);
int eb_screen_timing(eb_engine* e, double* total_ms, uint64_t* launches, uint64_t* rows);

/* ---------------------------------------------------------------- buffers */

/* Device::zeros_f32 / zeros_u32 (core/mod.rs:84-85): a zeroed buffer of `len`
 * elements of `dtype`. */
int eb_buf_alloc(eb_engine* e, int dtype, size_t len, eb_buf** out);
/* A non-owning view of `len` elements of device memory at `dev_ptr` (on the
 * engine's device; 16-byte aligned). The memory must outlive the view. */
int eb_buf_wrap(eb_engine* e, int dtype, void* dev_ptr, size_t len, eb_buf** out);
int eb_buf_free(eb_engine* e, eb_buf* b);
size_t eb_buf_len(const eb_buf* b);
void* eb_buf_ptr(const eb_buf* b);
/* Device::write_f32 / write_u32 (core/mod.rs:86-88): overwrite
 * b[offset .. offset+len) from host memory, after queued work that uses b. */
int eb_buf_write(eb_engine* e, eb_buf* b, size_t offset, const void* host, size_t len);
/* Device::read_f32 / read_u32 (core/mod.rs:89-91): wait, copy b[lo..hi) to host. */
int eb_buf_read(eb_engine* e, const eb_buf* b, size_t lo, size_t hi, void* host);
/* Device::upload_f32 / upload_u32 (core/mod.rs:82-83). */
int eb_buf_upload(eb_engine* e, int dtype, const void* host, size_t len, eb_buf** out);
/* Device::bind (core/mod.rs:79-81): put the n x d data set on the device. The
 * engine also keeps the data's row norms and its FP16 screen copy for top-1. */
int eb_bind(eb_engine* e, const float* x, size_t n, size_t d, eb_buf** out);

/* ---------------------------------------------------------------- layer-1 ops */

/* Device::top1 (core/mod.rs:97-112). For every selection position p in
 * r0..r1, row x[ids[p]] (or x[p] when ids is NULL) gets labels[p] = best of
 * the k centroids and scores[p] its score. cnorm (k squared norms) is
 * required for EB_L2. */
int eb_top1(eb_engine* e, const eb_buf* x, size_t d, const eb_buf* ids, size_t r0, size_t r1,
            const eb_buf* centroids, const eb_buf* cnorm, size_t k, int metric, eb_buf* labels,
            eb_buf* scores);

/* Device::topk (core/mod.rs:114-124): the best kk (1..=16) data rows of every
 * query by inner product, best first (larger score, then lower id). With
 * exclude_self, query i is data row i and is skipped. Missing neighbours:
 * id 0xFFFFFFFF, score -inf. ids and sims are m*kk host arrays. */
int eb_topk(eb_engine* e, const float* queries, size_t m, const float* data, size_t n, size_t d,
            size_t kk, int exclude_self, uint32_t* ids, float* sims);

/* Device::scatter_add (core/mod.rs:126-139): sums (k x d) = the selected rows
 * added per label in selection order, counts (k) = rows per label; both are
 * overwritten. labels are read at positions r0..r1. With acc, acc += sums. */
int eb_scatter_add(eb_engine* e, const eb_buf* x, size_t d, const eb_buf* ids, size_t r0,
                   size_t r1, const eb_buf* labels, size_t k, eb_buf* sums, eb_buf* counts,
                   eb_buf* acc);

/* Device::row_norms (core/mod.rs:141-142): squared norm of each of `rows` rows. */
int eb_row_norms(eb_engine* e, const eb_buf* m, size_t rows, size_t d, eb_buf* out);

/* Device::normalize_rows (core/mod.rs:144-151): faiss normalize_into. */
int eb_normalize_rows(eb_engine* e, const eb_buf* src, size_t rows, size_t d, eb_buf* dst);

/* Device::split (core/mod.rs:153-162): apply a revival plan of npairs
 * (donor, dead) pairs (2*npairs host u32). The pairs must not share ids. */
int eb_split(eb_engine* e, eb_buf* positions, eb_buf* usage, const uint32_t* pairs,
             size_t npairs, size_t d);

/* Device::ema_update (core/mod.rs:164-177) with EmaStep{alpha, decay, replace}
 * (core/mod.rs:182-197). */
int eb_ema_update(eb_engine* e, eb_buf* positions, eb_buf* usage, const eb_buf* sums,
                  const eb_buf* counts, size_t k, size_t d, float alpha, float decay,
                  int replace);

/* ---------------------------------------------------------------- Assigner */

/* Assigner::bind_data / unbind_data (assign.rs:75-95): keep `data` (n x d) on
 * the device; eb_assign calls with ids into the same (pointer, n) then send
 * only the ids. Binding always takes a fresh copy. */
int eb_bind_data(eb_engine* e, const float* data, size_t n, size_t d);
int eb_unbind_data(eb_engine* e);

/* Assigner::assign (assign.rs:104-116; core::assign_on core/mod.rs:249-330).
 * ids == NULL: Rows::Dense, `rows` is n x d and m == n.
 * ids != NULL: Rows::Indexed{data: rows (n x d), ids (m)}.
 * centroids: k x d host. labels, scores: m host. */
int eb_assign(eb_engine* e, const float* rows, size_t n, size_t d, const uint32_t* ids,
              size_t m, const float* centroids, size_t k, int metric, uint32_t* labels,
              float* scores);

/* ---------------------------------------------------------------- Engine::run_train */

/* core::train::Job (core/train.rs:33-49) plus the recipe inputs of
 * model::Config (model.rs:23-67). */
typedef struct {
  const float* x; /* n x d host rows */
  size_t n, d, k;
  double nepochs;
  int32_t batch_law;     /* 0 auto, 1 throughput, 2 quality */
  int32_t spherical;     /* inner product on the unit sphere */
  int64_t batch_size;    /* 0: batch law */
  double alpha0;         /* NaN: step law */
  double unused_threshold; /* NaN: 0.1, or 0 when d <= 2 */
  uint32_t seed;
  int32_t capture;       /* fill labels */
  int64_t chunk;         /* rows per top-1 call; 0: 65536 */
  const float* init;     /* k x d initial centroids, or NULL: MT19937 draw */
  const float* state_positions; /* resume from EMA state (k x d), or NULL */
  const float* state_usage;     /* k, with state_positions */
  int32_t verbose;
} eb_train_job;

/* core::train::Outcome (core/train.rs:51-58) + model::EpochStats (model.rs:77-89). */
typedef struct {
  float* centroids; /* k x d */
  float* positions; /* k x d, may be NULL */
  float* usage;     /* k, may be NULL */
  int32_t* labels;  /* n, may be NULL */
  double obj[64];
  double imbalance[64];
  int64_t nsplit[64];
  double epoch_time[64];
  int32_t n_epochs;
  int64_t n_splits;
  int64_t batch_size;
  double alpha0;
  int64_t total_steps;
} eb_train_out;

int eb_train(eb_engine* e, const eb_train_job* job, eb_train_out* out);

/* ---------------------------------------------------------------- multi-GPU groups */

/* No counterpart in the reference (its engine is one device). Engines on
 * several GPUs, one per process or thread, form a group over NCCL: rank 0
 * calls eb_group_unique_id, the host hands the id to every rank by its own
 * means, and every rank calls eb_engine_join with it (collectively; it blocks
 * until all ranks joined). eb_train on a joined engine splits each batch's
 * top-1 across the ranks and all-gathers the labels and scores, so every rank
 * computes the same model as one engine alone, bit for bit; all ranks must
 * call it with the same job. NCCL is loaded when a group is formed. The group
 * is left when the engine is destroyed. */
#define EB_GROUP_ID_BYTES 128
int eb_group_unique_id(unsigned char* id);
int eb_engine_join(eb_engine* e, int rank, int world, const unsigned char* id);
int eb_engine_group(eb_engine* e, int* rank, int* world);
/* No counterpart in the reference. How eb_train on a joined engine divides a
 * batch (the data-parallel step of core/train.rs:60-303 over several GPUs):
 *  0 (default) splits its top-1 across the ranks only when the screen time
 *    that saves (its length in 128-row x 256-centroid tile times, about
 *    0.52 us per 64 columns of d each) exceeds about 40 us, the cost of the
 *    exchange; otherwise every rank scores the batch whole, with no
 *    exchange (a C2 batch, 16,384 rows with k = 1024, is not split). 1
 *    always splits it; 2 never does. Modes 0-2 give the model of one engine
 *    alone, bit for bit.
 *  3 splits the top-1 and the scatter-add: each rank sums its slice's rows
 *    into partial k x d sums and k counts, one all-gather per step carries
 *    every rank's slice results and partials, and every rank adds the
 *    partials in rank order. All ranks get the same model, deterministic for
 *    a given group size, but the sums are not added in the single engine's
 *    row order, so the model agrees with it to rounding, not bit for bit.
 * All ranks must use the same mode. */
int eb_set_group_shard(eb_engine* e, int mode);

/* No counterpart in the reference. In-place all-gather over the engine's group
 * (NCCL, on the engine's stream): rank r's share is b[r * words_per_rank ..
 * (r + 1) * words_per_rank) of 32-bit words; afterwards every rank holds every
 * share. Collective: all ranks call it with the same words_per_rank. With a
 * sharded assign (each rank's eb_top1 over its rows r * s .. (r + 1) * s of
 * labels and scores) it gives every rank the labels and scores of all rows.
 * A no-op on an engine that is not in a group. */
int eb_group_allgather(eb_engine* e, eb_buf* b, size_t words_per_rank);

/* No counterpart in the reference. Collective: all ranks call it with the
 * same words. A buffer of `words` 32-bit words in the group's exchange
 * region: one allocation per rank, mapped on every other rank through CUDA
 * IPC. eb_group_allgather on this buffer (the whole of it, words_per_rank a
 * multiple of 4) pushes each rank's share straight into every peer's copy
 * over NVLink in one kernel (an entry and an exit round of flags, every wait
 * bounded: a peer that does not arrive within 2 s is reported as EB_ERROR at
 * the next sync) instead of NCCL. The region is the engine's: the buffer is a
 * view, valid until a larger region is requested or the group is left, and
 * eb_buf_free releases only the view. Alone, or when any rank cannot map the
 * regions (the ranks agree), a plain device buffer (NCCL serves the
 * all-gather). */
int eb_group_exchange(eb_engine* e, size_t words, eb_buf** out);
/* No counterpart in the reference. Whether the engine's exchange region is
 * mapped (1) or its all-gathers go through NCCL (0), and in `why` (cap bytes,
 * NUL-terminated; may be null) the reason the last set-up mapped none. */
int eb_group_exchange_info(eb_engine* e, int* mapped, char* why, size_t cap);

/* Device::topk over a database sharded across a group (knn_self over several
 * GPUs, crates/emeans-cluster/src/knn.rs:17-64): every rank passes the same m
 * queries and its own shard, rows shard_offset .. shard_offset + n_shard of an
 * n_total-row database; each ranks its shard (global ids), the lists are
 * all-gathered over NCCL and merged on the device by (larger score, then lower
 * id), so every rank gets the top-kk of eb_topk over the whole database. With
 * exclude_self, query i is database row i. Collective: all ranks call it. On
 * an engine that is not in a group it ranks the one shard alone. */
int eb_topk_group(eb_engine* e, const float* queries, size_t m, const float* shard,
                  size_t n_shard, size_t shard_offset, size_t n_total, size_t d, size_t kk,
                  int exclude_self, uint32_t* ids, float* sims);

/* ---------------------------------------------------------------- no-alloc top-1 */

/* No counterpart in the reference: its CPU path has no device memory to
 * allocate. The exact top-1 of eb_top1 (the SIMT kernel, same labels and
 * scores bit for bit) over raw device pointers, for callers that may not
 * allocate device memory during a call (a fixed per-request memory
 * footprint, no allocation pauses on a latency budget). Its one scratch, the
 * L2 row norms of the selection, is a fixed device array of
 * EB_NOALLOC_MAX_ROWS floats per device; larger selections are rejected with
 * EB_INVALID_ARGUMENT. x is n x d (rows x[ids[p]] or x[p]), c is k x d,
 * cnorm k squared norms (EB_L2 only), labels and scores are indexed by
 * position p in r0..r1; pointer sizes are the caller's to guarantee. The
 * first call on a device sets up the scratch's address and must come before
 * any stream capture. The array is shared by all engines on a device: calls
 * in flight at the same time on one device race; calls on one stream do not.
 * Asynchronous on the engine's stream; errors found on the device surface at
 * the next eb_sync. */
#define EB_NOALLOC_MAX_ROWS 1048576
int eb_top1_exact_noalloc(eb_engine* e, const float* x, size_t n, size_t d,
                          const uint32_t* ids, size_t r0, size_t r1, const float* c,
                          const float* cnorm, size_t k, int metric, uint32_t* labels,
                          float* scores);

/* ---------------------------------------------------------------- dedup */

/* dedup::DedupConfig (crates/emeans-cluster/src/dedup.rs:39-62). */
typedef struct {
  size_t k;              /* neighbours searched per row; 1 ..= 16 on this engine */
  float sim_threshold;   /* cosine at or above which two rows link, in [-1, 1] */
  float rep_threshold;   /* cosine to the star's anchor to stay; NaN: sim_threshold */
  double max_gap_secs;   /* largest time gap of a link; NaN: no time rule */
} eb_dedup_config;

/* dedup::DedupResult (dedup.rs:77-96). The caller provides every array with
 * room for n entries; the first n_groups entries of representatives, anchors
 * and sizes are written. */
typedef struct {
  uint32_t* group_of;        /* n: group of every row (groups by lowest row) */
  uint32_t* representatives; /* the row that stands for each group */
  uint32_t* anchors;         /* each group's star center */
  uint32_t* sizes;           /* members per group */
  float* nn_sim;             /* n: similarity to the nearest other row */
  uint64_t n_groups;
  uint64_t linked_pairs;     /* links that passed (each pair once) */
  uint64_t split_components; /* components the star cover cut */
} eb_dedup_out;

/* dedup::dedup_with_neighbors (dedup.rs:186-358), host code: near-duplicate
 * groups of the n x d unit rows x from their self-join neighbours (ids, sims:
 * n x kk, best first, 0xFFFFFFFF / -inf padding, the row itself excluded).
 * created_unix (n, NaN = unknown), burst (n, 0xFFFFFFFF = no burst) and
 * priority (n, not NaN) are optional (NULL). Bursts are always one group;
 * links need sim >= sim_threshold (and the time rule); each component is cut
 * into stars around the best-linked rows; the representative is the member of
 * highest priority, then highest mean similarity, then lowest id. Dots are
 * f32 products added in column order, as the reference's. Needs no device. */
int eb_dedup_with_neighbors(const float* x, size_t n, size_t d, const uint32_t* ids,
                            const float* sims, size_t kk, const double* created_unix,
                            const uint32_t* burst, const float* priority,
                            const eb_dedup_config* cfg, eb_dedup_out* out);

/* dedup::dedup (dedup.rs:160-183): the exact kNN self-join on the engine
 * (eb_topk, min(k, n - 1) neighbours) followed by eb_dedup_with_neighbors. */
int eb_dedup(eb_engine* e, const float* x, size_t n, size_t d, const double* created_unix,
             const uint32_t* burst, const float* priority, const eb_dedup_config* cfg,
             eb_dedup_out* out);

/* ---------------------------------------------------------------- metrics */

/* metrics::Internal (crates/emeans-cluster/src/metrics.rs:94-112). */
typedef struct {
  uint64_t k_eff;           /* non-empty clusters */
  double silhouette;        /* mean cosine-distance silhouette; 0 when k_eff < 2 */
  double calinski_harabasz; /* variance ratio on the rows (Euclidean) */
  double davies_bouldin;    /* Davies-Bouldin index on the rows (Euclidean) */
  double objective;         /* mean 2 - 2 cos to the normalised cluster sum */
} eb_internal;

/* metrics::internal_scores (metrics.rs:115-274), the metrics' gemm_nt
 * (crates/emeans-core/src/assign.rs:813-825) on the device: rows x (n x d
 * host, unit rows), labels (n host, each < k). Cluster sums in f64 in row
 * order and every per-row, per-cluster and final formula in the reference's
 * f64 order; the n x k_eff products are FP32 FMA chains (the reference's
 * gemm crate adds in its own order, so results agree to rounding, not
 * bitwise). Rows bound with eb_bind_data (the same host pointer) are used in
 * place. sizes: k counts out, or NULL. */
int eb_internal_scores(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* labels,
                       size_t k, eb_internal* out, uint64_t* sizes);

#ifdef __cplusplus
}
#endif
#endif /* EMEANS_B200_H */
