/*
 * CPU oracle for the emeans hot path: TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C++, the float order of the reference's CPU
 * path (crate emeans-core): the MT19937 streams, the recipe, the fused top-1
 * (one sequential FMA chain per dot), the row-ordered scatter-add, the EMA
 * step, normalisation, revival and the device training loop. It is the
 * checker that the CUDA engine is compared against, and the timed CPU
 * baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it; the product library never links or calls it.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function here against
 * golden vectors produced by running the reference's own Python
 * implementation (reference/faiss_e_means, see tests/golden/make_golden.py)
 * and against the reference's committed fixture file when it is present.
 *
 * All functions are extern "C" with plain pointers. Return codes: 0 ok,
 * 1 invalid argument (message in orc_last_error()).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* orc_last_error(void);

/* ---- MT19937 (crates/emeans-core/src/rng.rs:13-103) ---- */
void orc_permutation(uint32_t seed, size_t n, uint32_t* out);
void orc_random_sample(uint32_t seed, size_t count, double* out);

/* ---- recipe (crates/emeans-core/src/recipe.rs:171-268) ---- */
enum { ORC_LAW_AUTO = 0, ORC_LAW_THROUGHPUT = 1, ORC_LAW_QUALITY = 2 };
typedef struct {
  int64_t batch_size;
  double alpha0;
  int32_t resolved_law; /* 1 throughput, 2 quality, 0 when the batch was given */
  int32_t n_epochs;
  int64_t steps_per_pass;
  int64_t total_steps;
  int64_t epoch_rows[64];
  int64_t epoch_steps[64];
} orc_recipe_t;
/* batch_size 0 = not given; alpha0 NaN = not given. */
int orc_recipe(size_t n, size_t k, size_t d, double nepochs, int law, size_t batch_size,
               double alpha0, orc_recipe_t* out);
double orc_scheduled_alpha(double alpha0, size_t step, size_t total_steps);
double orc_unused_threshold(double given_or_nan, size_t d);
uint32_t orc_epoch_seed(uint32_t seed, size_t epoch);

/* ---- layer-1 ops (crates/emeans-core/src/core/cpu.rs, assign.rs, assign/fused.rs) ---- */
enum { ORC_L2 = 0, ORC_IP = 1 };
void orc_row_norms(const float* m, size_t rows, size_t d, float* out);
void orc_normalize_rows(const float* src, size_t rows, size_t d, float* dst);
/* Rows r0..r1 of the selection (x[ids[p]] or x[p]); outputs at positions p. */
int orc_top1(const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0, size_t r1,
             const float* c, size_t k, int metric, uint32_t* labels, float* scores,
             int threads);
int orc_scatter_add(const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0,
                    size_t r1, const uint32_t* labels, size_t k, float* sums,
                    uint32_t* counts, float* acc);
void orc_ema_update(float* pos, float* usage, const float* sums, const uint32_t* counts,
                    size_t k, size_t d, float alpha, float decay, int replace);
/* pairs: npairs (donor, dead) u32 pairs, applied in order. */
void orc_split(float* pos, float* usage, size_t k, size_t d, const uint32_t* pairs,
               size_t npairs);
float orc_numpy_sum_f32(const float* a, size_t n);
/* Revival plan with an RNG that lives across calls. */
void* orc_rng_new(uint32_t seed);
void orc_rng_free(void* rng);
size_t orc_plan_revival(const float* usage, size_t k, double tau, void* rng,
                        uint32_t* pairs_out);
void orc_closing_means(const float* pos, const float* sums, const double* counts,
                       size_t k, size_t d, int spherical, float* out);

/* ---- exact top-k by inner product (FMA-chain scores; best first, lower id on ties) ---- */
int orc_topk(const float* q, size_t m, const float* data, size_t n, size_t d, size_t kk,
             int exclude_self, uint32_t* ids, float* sims, int threads);
// knn_self for the queries data[q0 .. q0 + m) only (each skips its own row).
int orc_topk_self_rows(const float* data, size_t n, size_t d, size_t q0, size_t m, size_t kk,
                       uint32_t* ids, float* sims, int threads);

/* ---- layer 2: the training loop (crates/emeans-core/src/core/train.rs:60-303) ---- */
typedef struct {
  double nepochs;
  int32_t batch_law;
  int32_t spherical;
  int64_t batch_size;      /* 0 = batch law */
  double alpha0;           /* NaN = step law */
  double unused_threshold; /* NaN = default */
  uint32_t seed;
  int32_t capture;
  int64_t chunk; /* 0 = 65536 */
  int32_t threads;
} orc_train_cfg;
typedef struct {
  float* centroids;  /* k*d */
  float* positions;  /* k*d */
  float* usage;      /* k */
  int32_t* labels;   /* n, may be NULL */
  double obj[64];
  double imbalance[64];
  int64_t nsplit[64];
  int32_t n_epochs;
  int64_t n_splits;
  int64_t batch_size;
  double alpha0;
} orc_train_out;
/* init: k*d initial centroids or NULL (MT19937 draw); state_pos/state_usage: resume
 * from EMA state (both or neither). */
int orc_train(const float* x, size_t n, size_t d, size_t k, const orc_train_cfg* cfg,
              const float* init, const float* state_pos, const float* state_usage,
              orc_train_out* out);

#ifdef __cplusplus
}
#endif
