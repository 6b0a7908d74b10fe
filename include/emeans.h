/*
 * emeans.h for libemeans.so built by emeans_b200: the reference's C FFI
 * (crates/emeans-ffi/include/emeans.h, crates/emeans-ffi/src/lib.rs) for its
 * assign call, on the B200 engine.
 *
 * A C, Go (cgo) or Python (ctypes) program written against the reference's
 * header links this libemeans.so instead and keeps its calls: the names,
 * signatures, status codes, result handles and error rules below are the
 * reference's. Only the subset listed here is provided; the model, hierarchy,
 * dedup and one-shot train calls of the reference header are not in this
 * library (a program that uses them does not link against it).
 *
 * Differences, by design:
 *  - `backend` NULL selects this library's one backend, the B200 engine on the
 *    calling thread's current CUDA device (the reference's default is "cpu").
 *    "cuda", "cuda-fused" and "b200" name it too; the reference's other
 *    backend names are EMEANS_ERROR ("not in this library").
 *  - There is no CPU fallback: with no usable GPU, emeans_assign is
 *    EMEANS_ERROR.
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
