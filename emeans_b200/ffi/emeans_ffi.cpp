// libemeans.so: the reference's C FFI for its assign call
// (crates/emeans-ffi/src/lib.rs), answered by the B200 engine through the
// emeans_b200 C ABI. Host code only; it links against libemeans_b200.so.
//
// The error rules follow the reference's boundary: every call but
// emeans_last_error clears the thread's message first (lib.rs:124-147);
// out-pointers are checked before any work (lib.rs:213-219); a NULL array
// with a non-zero length, a size that overflows or a misaligned pointer is
// EMEANS_INVALID_ARGUMENT (lib.rs:149-174); shape, metric and backend
// failures are EMEANS_ERROR in the order bindings/common/src/lib.rs:327-346
// checks them; an unexpected exception is EMEANS_PANIC.
#include "emeans.h"

#include <stdint.h>

#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "emeans_b200.h"

namespace {

thread_local std::string t_error;
thread_local bool t_failed = false;

struct BadArg : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct Refused : std::runtime_error {
  using std::runtime_error::runtime_error;
};

template <class F>
int32_t guard(F&& f) {
  t_failed = false;
  t_error.clear();
  try {
    f();
    return EMEANS_OK;
  } catch (const BadArg& e) {
    t_error = e.what();
    t_failed = true;
    return EMEANS_INVALID_ARGUMENT;
  } catch (const Refused& e) {
    t_error = e.what();
    t_failed = true;
    return EMEANS_ERROR;
  } catch (const std::bad_alloc&) {
    t_error = "out of host memory";
    t_failed = true;
    return EMEANS_ERROR;
  } catch (const std::exception& e) {
    t_error = std::string("panic in emeans: ") + e.what();
    t_failed = true;
    return EMEANS_PANIC;
  } catch (...) {
    t_error = "panic in emeans: unknown exception";
    t_failed = true;
    return EMEANS_PANIC;
  }
}

size_t mul(size_t a, size_t b) {
  size_t r;
  if (__builtin_mul_overflow(a, b, &r)) throw BadArg("n * d overflows");
  return r;
}

template <class T>
void check_slice(const T* p, size_t len, const char* what) {
  if (len == 0) return;
  if (!p) throw BadArg(std::string(what) + " is NULL");
  if (reinterpret_cast<uintptr_t>(p) % alignof(T) != 0) throw BadArg(std::string(what) + " is not aligned");
}

const char* need_string(const char* p, const char* what) {
  if (!p) throw BadArg(std::string(what) + " is NULL");
  return p;
}

int parse_metric(const std::string& m) {
  if (m == "l2") return EB_L2;
  if (m == "inner_product" || m == "ip" || m == "cosine") return EB_IP;
  throw Refused("unknown metric \"" + m + "\" (l2, inner_product)");
}

// The reference's backend names (crates/emeans-cluster/src/backend.rs:72-101).
void check_backend(const char* b) {
  if (!b) return;
  const std::string s(b);
  if (s == "cuda" || s == "cuda-fused" || s == "b200") return;
  static const char* known[] = {"cpu",   "cpu-blocked", "cpu-gemm",  "cpu-accelerate",
                                "cpu-fused", "metal",   "metal-fused", "cuda-bf16"};
  for (const char* k : known)
    if (s == k) throw Refused("backend \"" + s + "\" is not in this library (it runs: cuda, b200)");
  throw Refused("unknown backend \"" + s + "\" (this library runs: cuda, b200)");
}

// One engine for the process, on device EMEANS_B200_DEVICE (default 0),
// created on first use and used by one call at a time.
std::mutex g_mu;
eb_engine* g_engine = nullptr;

eb_engine* engine_locked() {
  if (g_engine) return g_engine;
  int dev = 0;
  if (const char* s = std::getenv("EMEANS_B200_DEVICE")) dev = std::atoi(s);
  eb_engine* e = nullptr;
  if (eb_engine_create(dev, &e) != EB_OK) throw Refused(std::string("no B200 engine: ") + eb_last_error());
  g_engine = e;
  return e;
}

}  // namespace

struct EmeansResult {
  std::vector<uint32_t> labels;
  std::vector<float> scores;
  std::string json = "{}";
};

extern "C" {

uint32_t emeans_abi_version(void) { return EMEANS_ABI_VERSION; }

const char* emeans_version(void) { return "0.1.0"; }

const char* emeans_last_error(void) { return t_failed ? t_error.c_str() : nullptr; }

void emeans_string_free(char* s) { std::free(s); }

int32_t emeans_backends(char** out_json) {
  return guard([&] {
    if (!out_json) throw BadArg("out_json is NULL");
    bool ok = false;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      try {
        engine_locked();
        ok = true;
      } catch (const Refused&) {
      }
    }
    const char* v = ok ? "[\"cuda\"]" : "[]";
    char* s = static_cast<char*>(std::malloc(std::strlen(v) + 1));
    if (!s) throw std::bad_alloc();
    std::strcpy(s, v);
    *out_json = s;
  });
}

int32_t emeans_assign(const float* data, size_t n, size_t d, const float* centroids, size_t k,
                      const char* metric, const char* backend, EmeansResult** out_result) {
  return guard([&] {
    if (!out_result) throw BadArg("out_result is NULL");
    check_slice(data, mul(n, d), "data");
    check_slice(centroids, mul(k, d), "centroids");
    const std::string m(need_string(metric, "metric"));
    if (d == 0) throw Refused("d must be positive");
    if (k == 0) throw Refused("centroids is empty");
    const int met = parse_metric(m);
    check_backend(backend);
    std::unique_ptr<EmeansResult> r(new EmeansResult);
    r->labels.resize(n);
    r->scores.resize(n);
    if (n > 0) {
      std::lock_guard<std::mutex> lk(g_mu);
      eb_engine* e = engine_locked();
      const int rc = eb_assign(e, data, n, d, nullptr, n, centroids, k, met, r->labels.data(),
                               r->scores.data());
      if (rc == EB_INVALID_ARGUMENT) throw Refused(eb_last_error());
      if (rc != EB_OK) throw Refused(std::string("device: ") + eb_last_error());
    }
    *out_result = r.release();
  });
}

int32_t emeans_result_array(const EmeansResult* r, const char* name, EmeansArray* out_array) {
  return guard([&] {
    if (!r) throw BadArg("result is NULL");
    const std::string nm(need_string(name, "name"));
    EmeansArray a;
    if (nm == "labels") {
      a = {r->labels.empty() ? nullptr : r->labels.data(), r->labels.size(), EMEANS_U32};
    } else if (nm == "scores") {
      a = {r->scores.empty() ? nullptr : r->scores.data(), r->scores.size(), EMEANS_F32};
    } else {
      throw Refused("the result has no array \"" + nm + "\" (has: labels, scores)");
    }
    if (!out_array) throw BadArg("out_array is NULL");
    *out_array = a;
  });
}

const char* emeans_result_json(const EmeansResult* r) { return r ? r->json.c_str() : nullptr; }

void emeans_result_free(EmeansResult* r) { delete r; }

}  // extern "C"
