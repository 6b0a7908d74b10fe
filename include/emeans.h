/*
 * emeans.h for libemeans.so built by emeans_b200: the reference's C FFI
 * (crates/emeans-ffi/include/emeans.h, crates/emeans-ffi/src/lib.rs) for its
 * assign, train and in-memory model calls, on the B200 engine.
 *
 * A C, Go (cgo) or Python (ctypes) program written against the reference's
 * header links this libemeans.so instead and keeps its calls: the names,
 * signatures, status codes, result handles and error rules below are the
 * reference's. Only the subset listed here is provided; model files and bytes
 * (save, load, to/from bytes), the hierarchy, auto-clustering and dedup calls
 * of the reference header are not in this library (a program that uses them
 * does not link against it).
 *
 * Differences, by design:
 *  - `backend` NULL (and a config without "backend") selects this library's
 *    one backend, the B200 engine on device EMEANS_B200_DEVICE (environment,
 *    default 0). "cuda", "cuda-fused" and "b200" name it too, and so do
 *    "cpu" (the reference's default, its fused kernel on x86_64) and
 *    "cpu-fused": the engine returns that kernel's results bit for bit. The
 *    reference's other backend names (other float orders) are EMEANS_ERROR
 *    ("not in this library").
 *  - There is no CPU fallback: with no usable GPU, every call that computes
 *    is EMEANS_ERROR.
 *  - Result JSON numbers are written with 17 significant digits (the same
 *    doubles as the reference's shortest form).
 * Results are bit-equal to the reference's CPU assign (`cpu-fused` order:
 * one FMA chain per dot, ties to the lower id).
 */
#ifndef EMEANS_H
#define EMEANS_H

#include <stddef.h>
#include <stdint.h>

/* emeans.h:63 */
#define EMEANS_ABI_VERSION 1

/* Status codes, emeans.h:66-80. */
#define EMEANS_OK 0
#define EMEANS_INVALID_ARGUMENT 1 /* NULL with a non-zero length, overflow, misalignment */
#define EMEANS_ERROR 2            /* bad shape or metric, unknown backend, device failure */
#define EMEANS_PANIC 3            /* an unexpected exception caught at the boundary */

/* Element types of an EmeansArray, emeans.h:83-92. */
#define EMEANS_F32 0
#define EMEANS_U32 1
#define EMEANS_I32 2
#define EMEANS_U8 3

/* emeans.h:106-109: named arrays and a JSON object of scalars; caller-owned. */
typedef struct EmeansResult EmeansResult;

/* emeans.h:101-104: a trained model (its centroids and metric), in memory. */
typedef struct EmeansModel EmeansModel;

/* emeans.h:114-121: a borrowed view into a result. */
typedef struct EmeansArray {
  const void *data; /* NULL when len is 0 */
  size_t len;       /* elements, not bytes */
  int32_t dtype;    /* EMEANS_F32, EMEANS_U32, EMEANS_I32 or EMEANS_U8 */
} EmeansArray;

#ifdef __cplusplus
extern "C" {
#endif

/* emeans.h:129 (lib.rs:281). Always EMEANS_ABI_VERSION. */
uint32_t emeans_abi_version(void);

/* emeans.h:132 (lib.rs:287). "major.minor.patch"; static, do not free. */
const char *emeans_version(void);

/* emeans.h:137 (lib.rs:295). The calling thread's last failure message, or
 * NULL when its last emeans call succeeded. Every call except this one
 * clears it first. */
const char *emeans_last_error(void);

/* emeans.h:142 (lib.rs:303). Frees a string returned through a char**. */
void emeans_string_free(char *s);

/* emeans.h:153 (lib.rs:331). JSON array of the backend names this library
 * can run on this machine: ["cuda"] with a usable GPU, [] without.
 * Free *out_json with emeans_string_free. */
int32_t emeans_backends(char **out_json);

/* emeans.h:144-147 (lib.rs:315-323). The default config of kind "train" as
 * JSON ("backend": "cuda"); "auto" and "dedup" are EMEANS_ERROR here. Free
 * *out_json with emeans_string_free. */
int32_t emeans_default_config(const char *kind, char **out_json);

/* emeans.h:155-179 (lib.rs:361-378, bindings/common/src/lib.rs:189-231).
 * Trains k centroids on data (n * d floats) with the reference's device loop
 * (bit-equal to the reference's CPU training with the same config).
 * config_json: overrides of emeans_default_config("train") or NULL; keys
 * nepochs, batch_size, alpha0, batch_law, seed, spherical, unused_threshold,
 * max_points_per_centroid, assignment_chunk_size, capture_assignments,
 * verbose, exact_objective, backend. Result arrays: "centroids" (EMEANS_F32,
 * k * d) and, with capture_assignments, "labels" (EMEANS_I32, n; -1 outside
 * the training subset). Result JSON: k, d, objective, exact_objective, stats
 * (obj, time, imbalance_factor, nsplit per epoch), backend. */
int32_t emeans_train(const float *data, size_t n, size_t d, size_t k, const char *config_json,
                     EmeansResult **out_result);

/* emeans.h:214-225 (lib.rs:457-480). emeans_train that also returns the
 * model; out_result may be NULL. Free the model with emeans_model_free. */
int32_t emeans_model_train(const float *data, size_t n, size_t d, size_t k,
                           const char *config_json, EmeansModel **out_model,
                           EmeansResult **out_result);

/* emeans.h:227-234 (lib.rs:484-499). The model's nearest centroid for each
 * row (n * d floats): inner product when spherical, else squared L2. Result
 * arrays as emeans_assign. */
int32_t emeans_model_assign(const EmeansModel *m, const float *data, size_t n,
                            EmeansResult **out_result);

/* emeans.h:236-242 (lib.rs:503-517). Mean squared distance, or mean 2 - 2 cos
 * when spherical, of the rows to their nearest centroid. */
int32_t emeans_model_objective(const EmeansModel *m, const float *data, size_t n,
                               double *out_objective);

/* emeans.h:244-248 (lib.rs:521-534). A view of the k * d centroids, valid
 * until the model is freed. */
int32_t emeans_model_centroids(const EmeansModel *m, EmeansArray *out_array);

/* emeans.h:250-252 (lib.rs:539-548). JSON: d, k, metric, spherical, backend,
 * epochs. Free *out_json with emeans_string_free. */
int32_t emeans_model_info(const EmeansModel *m, char **out_json);

/* emeans.h:274-275 (lib.rs:620-625). NULL is a no-op. */
void emeans_model_free(EmeansModel *m);

/* emeans.h:189-196 (lib.rs:387-408, bindings/common/src/lib.rs:327-346).
 * The nearest of k centroids (k * d floats) for every row of data (n * d
 * floats). metric: "l2" (squared distance, smallest wins) or
 * "inner_product" / "ip" / "cosine" (largest wins). Result arrays: "labels"
 * (EMEANS_U32, n) and "scores" (EMEANS_F32, n); result JSON "{}". */
int32_t emeans_assign(const float *data, size_t n, size_t d, const float *centroids, size_t k,
                      const char *metric, const char *backend, EmeansResult **out_result);

/* emeans.h:339-341 (lib.rs:784-809). EMEANS_ERROR when the result has no
 * array of that name; the message lists the names it has. */
int32_t emeans_result_array(const EmeansResult *r, const char *name, EmeansArray *out_array);

/* emeans.h:345 (lib.rs:814). "{}" for an assign result; NULL for NULL. */
const char *emeans_result_json(const EmeansResult *r);

/* emeans.h:348 (lib.rs:821). NULL is a no-op. */
void emeans_result_free(EmeansResult *r);

#ifdef __cplusplus
}
#endif

#endif /* EMEANS_H */
