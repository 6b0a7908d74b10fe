// libemeans.so: the reference's C FFI (crates/emeans-ffi/src/lib.rs) for its
// assign, train and in-memory model calls, answered by the B200 engine through
// the emeans_b200 C ABI. Host code only; it links against libemeans_b200.so.
//
// The error rules follow the reference's boundary: every call but
// emeans_last_error clears the thread's message first (lib.rs:124-147);
// out-pointers are checked before any work (lib.rs:213-219); a NULL array
// with a non-zero length, a size that overflows, a misaligned pointer or a
// config that is not valid JSON is EMEANS_INVALID_ARGUMENT (lib.rs:149-201);
// shape, metric, config and backend failures are EMEANS_ERROR in the order
// bindings/common/src/lib.rs checks them; an unexpected exception is
// EMEANS_PANIC.
#include "emeans.h"

#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "emeans_b200.h"
#include "host.h"

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

char* new_cstring(const std::string& v) {
  char* s = static_cast<char*>(std::malloc(v.size() + 1));
  if (!s) throw std::bad_alloc();
  std::memcpy(s, v.c_str(), v.size() + 1);
  return s;
}

int parse_metric(const std::string& m) {
  if (m == "l2") return EB_L2;
  if (m == "inner_product" || m == "ip" || m == "cosine") return EB_IP;
  throw Refused("unknown metric \"" + m + "\" (l2, inner_product)");
}

// The reference's backend names (crates/emeans-cluster/src/backend.rs:72-101).
// "cpu" is the reference's default; on x86_64 it resolves to the fused kernel
// (CpuKernel::fastest, crates/emeans-core/src/assign.rs:250-260), whose float
// order (one FMA chain per dot, lower id on ties) this engine reproduces bit
// for bit, so "cpu" and "cpu-fused" are served here with identical results.
// The other CPU kernels, Metal and cuda-bf16 add in other orders: refused.
void check_backend(const std::string& s) {
  if (s == "cuda" || s == "cuda-fused" || s == "b200" || s == "cpu" || s == "cpu-fused") return;
  static const char* known[] = {"cpu-blocked", "cpu-gemm", "cpu-accelerate", "metal",
                                "metal-fused", "cuda-bf16"};
  for (const char* k : known)
    if (s == k)
      throw Refused("backend \"" + s + "\" is not in this library (it runs: cpu, cpu-fused, cuda, b200)");
  throw Refused("unknown backend \"" + s + "\" (this library runs: cpu, cpu-fused, cuda, b200)");
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

void engine_call(int rc) {
  if (rc != EB_OK) throw Refused(eb_last_error());
}

// ---- JSON: a reader for config overrides and a writer for result scalars.

struct Json {
  enum Kind { Null, Bool, Num, Str, Obj, Arr } kind = Null;
  bool b = false;
  double num = 0.0;
  bool integral = false;  // written without fraction or exponent
  std::string str;
  std::vector<std::pair<std::string, Json>> obj;
  std::vector<Json> arr;
};

struct Reader {
  const char* p;
  const char* end;
  [[noreturn]] void fail() { throw BadArg("config is not valid JSON"); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
  }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if ((size_t)(end - p) >= n && std::memcmp(p, s, n) == 0) {
      p += n;
      return true;
    }
    return false;
  }
  // The four hex digits of a \\u escape (p at the u); p ends on the last digit.
  unsigned hex4() {
    if (end - p < 5) fail();
    unsigned v = 0;
    for (int i = 1; i <= 4; i++) {
      const char c = p[i];
      v = v * 16 + (c >= '0' && c <= '9' ? c - '0'
                    : c >= 'a' && c <= 'f' ? c - 'a' + 10
                    : c >= 'A' && c <= 'F' ? c - 'A' + 10
                                           : (fail(), 0));
    }
    p += 4;
    return v;
  }
  std::string string() {
    if (p >= end || *p != '"') fail();
    p++;
    std::string out;
    while (p < end && *p != '"') {
      if ((unsigned char)*p < 0x20) fail();
      if (*p == '\\') {
        if (++p >= end) fail();
        switch (*p) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            unsigned v = hex4();
            // A UTF-16 surrogate pair is one code point; a lone surrogate is
            // not valid JSON text (serde_json refuses it too).
            if (v >= 0xDC00 && v <= 0xDFFF) fail();
            if (v >= 0xD800 && v <= 0xDBFF) {
              if (end - p < 7 || p[1] != '\\' || p[2] != 'u') fail();
              p += 2;
              const unsigned lo = hex4();
              if (lo < 0xDC00 || lo > 0xDFFF) fail();
              v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
            }
            // Config keys and values are ASCII; other code points keep their
            // UTF-8 form only for messages.
            if (v < 0x80) {
              out += (char)v;
            } else if (v < 0x800) {
              out += (char)(0xC0 | (v >> 6));
              out += (char)(0x80 | (v & 0x3F));
            } else if (v < 0x10000) {
              out += (char)(0xE0 | (v >> 12));
              out += (char)(0x80 | ((v >> 6) & 0x3F));
              out += (char)(0x80 | (v & 0x3F));
            } else {
              out += (char)(0xF0 | (v >> 18));
              out += (char)(0x80 | ((v >> 12) & 0x3F));
              out += (char)(0x80 | ((v >> 6) & 0x3F));
              out += (char)(0x80 | (v & 0x3F));
            }
            break;
          }
          default: fail();
        }
        p++;
      } else {
        out += *p++;
      }
    }
    if (p >= end) fail();
    p++;
    return out;
  }
  Json value(int depth) {
    if (depth > 64) fail();
    ws();
    if (p >= end) fail();
    Json v;
    if (*p == '{') {
      p++;
      v.kind = Json::Obj;
      ws();
      if (p < end && *p == '}') {
        p++;
        return v;
      }
      for (;;) {
        ws();
        std::string k = string();
        ws();
        if (p >= end || *p != ':') fail();
        p++;
        v.obj.emplace_back(k, value(depth + 1));
        ws();
        if (p < end && *p == ',') {
          p++;
          continue;
        }
        if (p < end && *p == '}') {
          p++;
          return v;
        }
        fail();
      }
    }
    if (*p == '[') {
      p++;
      v.kind = Json::Arr;
      ws();
      if (p < end && *p == ']') {
        p++;
        return v;
      }
      for (;;) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (p < end && *p == ',') {
          p++;
          continue;
        }
        if (p < end && *p == ']') {
          p++;
          return v;
        }
        fail();
      }
    }
    if (*p == '"') {
      v.kind = Json::Str;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Json::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Json::Bool;
      return v;
    }
    if (lit("null")) return v;
    // number: -?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][+-]?[0-9]+)?
    const char* s = p;
    if (p < end && *p == '-') p++;
    if (p >= end || !(*p >= '0' && *p <= '9')) fail();
    if (*p == '0') {
      p++;
    } else {
      while (p < end && *p >= '0' && *p <= '9') p++;
    }
    bool integral = true;
    if (p < end && *p == '.') {
      integral = false;
      p++;
      if (p >= end || !(*p >= '0' && *p <= '9')) fail();
      while (p < end && *p >= '0' && *p <= '9') p++;
    }
    if (p < end && (*p == 'e' || *p == 'E')) {
      integral = false;
      p++;
      if (p < end && (*p == '+' || *p == '-')) p++;
      if (p >= end || !(*p >= '0' && *p <= '9')) fail();
      while (p < end && *p >= '0' && *p <= '9') p++;
    }
    v.kind = Json::Num;
    v.integral = integral;
    v.num = std::strtod(std::string(s, p).c_str(), nullptr);
    return v;
  }
};

std::string fmt_num(double v) {
  if (!std::isfinite(v)) return "null";  // as serde_json writes non-finite floats
  char b[40];
  std::snprintf(b, sizeof b, "%.17g", v);
  std::string s(b);
  if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
  return s;
}

// ---- the train config (model::Config, crates/emeans-core/src/model.rs:23-67,
// and the FFI's defaults, bindings/common/src/lib.rs:36-57).

struct TrainConfig {
  double nepochs = 5.0;
  bool batch_size_set = false;
  uint64_t batch_size = 0;
  bool alpha0_set = false;
  double alpha0 = 0.0;
  int batch_law = 0;  // auto, throughput, quality
  uint32_t seed = 1234;
  bool spherical = false;
  bool tau_set = false;
  double unused_threshold = 0.0;
  bool mppc_set = false;
  uint64_t max_points_per_centroid = 0;
  bool chunk_set = false;
  uint64_t assignment_chunk_size = 0;
  bool capture_assignments = true;
  bool verbose = false;
  bool exact_objective = false;
  std::string backend = "cuda";
};

const char* kTrainKeys[] = {"alpha0",         "assignment_chunk_size", "backend",
                            "batch_law",      "batch_size",            "capture_assignments",
                            "exact_objective", "max_points_per_centroid", "nepochs",
                            "seed",           "spherical",             "unused_threshold",
                            "verbose"};

std::string default_train_config() {
  return "{\"alpha0\":null,\"assignment_chunk_size\":null,\"backend\":\"cuda\","
         "\"batch_law\":\"auto\",\"batch_size\":null,\"capture_assignments\":true,"
         "\"exact_objective\":false,\"max_points_per_centroid\":null,\"nepochs\":5.0,"
         "\"seed\":1234,\"spherical\":false,\"unused_threshold\":null,\"verbose\":false}";
}

[[noreturn]] void bad_config(const std::string& key, const char* want) {
  throw Refused("bad train config: \"" + key + "\" must be " + want);
}

uint64_t as_uint(const Json& v, const std::string& key, double max) {
  // (double)UINT64_MAX rounds up to 2^64, which does not convert: refused.
  if (v.kind != Json::Num || !v.integral || v.num < 0 || v.num > (double)max ||
      v.num >= 18446744073709551616.0)
    bad_config(key, "a non-negative integer");
  return (uint64_t)v.num;
}

double as_num(const Json& v, const std::string& key) {
  if (v.kind != Json::Num) bad_config(key, "a number");
  return v.num;
}

bool as_bool(const Json& v, const std::string& key, const char* want = "true or false") {
  if (v.kind != Json::Bool) bad_config(key, want);
  return v.b;
}

// parse_overrides (bindings/common/src/lib.rs:115-124): the config text as
// JSON, or null for NULL, empty or "null" text; invalid JSON is BadArg.
Json parse_overrides(const char* text) {
  Json root;
  if (!text) return root;
  Reader r{text, text + std::strlen(text)};
  r.ws();
  if (r.p == r.end) return root;
  root = r.value(0);
  r.ws();
  if (r.p != r.end) r.fail();
  return root;
}

// resolve (bindings/common/src/lib.rs:59-112): overrides over the defaults
// in the reference's order of checks: an object, no d or k, known keys,
// exact_objective a bool, backend a known name, then each field's type.
TrainConfig resolve_train_config(const Json& root) {
  TrainConfig c;
  if (root.kind == Json::Null) return c;
  if (root.kind != Json::Obj) throw Refused("config must be an object");
  for (const char* key : {"d", "k"})
    for (auto& kv : root.obj)
      if (kv.first == key)
        throw Refused(std::string("pass ") + key + " as an argument, not in the config");
  for (auto& kv : root.obj) {
    bool known = false;
    for (const char* name : kTrainKeys) known |= kv.first == name;
    if (!known) {
      std::string list;
      for (const char* name : kTrainKeys) list += std::string(list.empty() ? "" : ", ") + name;
      throw Refused("unknown config key \"" + kv.first + "\" (known: " + list + ")");
    }
  }
  for (auto& kv : root.obj)
    if (kv.first == "exact_objective") {
      if (kv.second.kind != Json::Bool)
        throw Refused("config key \"exact_objective\" must be true or false");
      c.exact_objective = kv.second.b;
    }
  for (auto& kv : root.obj)
    if (kv.first == "backend") {
      if (kv.second.kind != Json::Str) throw Refused("config key \"backend\" must be a string");
      c.backend = kv.second.str;
    }
  check_backend(c.backend);
  for (auto& kv : root.obj) {
    const std::string& k = kv.first;
    const Json& v = kv.second;
    if (k == "exact_objective" || k == "backend") {
      continue;
    } else if (k == "nepochs") {
      c.nepochs = as_num(v, k);
    } else if (k == "batch_size") {
      c.batch_size_set = v.kind != Json::Null;
      if (c.batch_size_set) c.batch_size = as_uint(v, k, (double)UINT64_MAX);
    } else if (k == "alpha0") {
      c.alpha0_set = v.kind != Json::Null;
      if (c.alpha0_set) c.alpha0 = as_num(v, k);
    } else if (k == "batch_law") {
      if (v.kind != Json::Str) bad_config(k, "\"auto\", \"throughput\" or \"quality\"");
      if (v.str == "auto") c.batch_law = 0;
      else if (v.str == "throughput") c.batch_law = 1;
      else if (v.str == "quality") c.batch_law = 2;
      else bad_config(k, "\"auto\", \"throughput\" or \"quality\"");
    } else if (k == "seed") {
      c.seed = (uint32_t)as_uint(v, k, 4294967295.0);
    } else if (k == "spherical") {
      c.spherical = as_bool(v, k);
    } else if (k == "unused_threshold") {
      c.tau_set = v.kind != Json::Null;
      if (c.tau_set) c.unused_threshold = as_num(v, k);
    } else if (k == "max_points_per_centroid") {
      c.mppc_set = v.kind != Json::Null;
      if (c.mppc_set) c.max_points_per_centroid = as_uint(v, k, (double)UINT64_MAX);
    } else if (k == "assignment_chunk_size") {
      c.chunk_set = v.kind != Json::Null;
      if (c.chunk_set) c.assignment_chunk_size = as_uint(v, k, (double)INT64_MAX);
    } else if (k == "capture_assignments") {
      c.capture_assignments = as_bool(v, k);
    } else if (k == "verbose") {
      c.verbose = as_bool(v, k);
    }
  }
  return c;
}

}  // namespace

struct EmeansResult {
  struct Array {
    std::string name;
    int32_t dtype;
    std::vector<float> f32;
    std::vector<uint32_t> u32;
    std::vector<int32_t> i32;
  };
  std::vector<Array> arrays;
  std::string json = "{}";
};

struct EmeansModel {
  size_t k = 0, d = 0;
  bool spherical = false;
  size_t epochs = 0;
  std::vector<float> centroids;
};

namespace {

std::unique_ptr<EmeansResult> assign_result(std::vector<uint32_t> labels, std::vector<float> scores) {
  std::unique_ptr<EmeansResult> r(new EmeansResult);
  r->arrays.resize(2);
  r->arrays[0].name = "labels";
  r->arrays[0].dtype = EMEANS_U32;
  r->arrays[0].u32 = std::move(labels);
  r->arrays[1].name = "scores";
  r->arrays[1].dtype = EMEANS_F32;
  r->arrays[1].f32 = std::move(scores);
  return r;
}

// Labels and scores of every row against k centroids (assign_all over the
// engine).
void run_assign(const float* data, size_t n, size_t d, const float* c, size_t k, int metric,
                std::vector<uint32_t>& labels, std::vector<float>& scores) {
  labels.assign(n, 0);
  scores.assign(n, 0.0f);
  if (n == 0) return;
  std::lock_guard<std::mutex> lk(g_mu);
  eb_engine* e = engine_locked();
  engine_call(eb_assign(e, data, n, d, nullptr, n, c, k, metric, labels.data(), scores.data()));
}

// AssignOutput::mean_objective (crates/emeans-core/src/model.rs:127-141).
double mean_objective(const std::vector<float>& scores, bool spherical) {
  double s = -0.0;
  for (float v : scores) s += spherical ? 2.0 - 2.0 * (double)v : (double)v;
  return s / (double)std::max<size_t>(scores.size(), 1);
}

// api::train_model (bindings/common/src/lib.rs:195-231) on the engine:
// Emeans::train_from's training subset (model.rs:704-770) and the device
// loop, then the result's arrays and JSON (lib.rs:153-187, ffi lib.rs:242-249).
void train_model(const float* data, size_t n, size_t d, size_t k, const char* config,
                 std::unique_ptr<EmeansModel>* model_out, std::unique_ptr<EmeansResult>* result_out) {
  const Json overrides = parse_overrides(config);  // invalid JSON: BadArg first (lib.rs:195-201)
  if (d == 0) throw Refused("d must be positive");
  if (k == 0) throw Refused("k must be positive");
  if (n < k) throw Refused("need at least k = " + std::to_string(k) + " rows, got " + std::to_string(n));
  const TrainConfig cfg = resolve_train_config(overrides);

  // Rows kept by max_points_per_centroid (model.rs:751-770).
  std::vector<uint32_t> keep;
  std::vector<float> sub;
  const float* x = data;
  size_t rows = n;
  if (cfg.mppc_set) {
    // A product past 2^64 - 1 keeps every row (the limit is above any n).
    uint64_t limit = 0;
    if (__builtin_mul_overflow(cfg.max_points_per_centroid, (uint64_t)k, &limit)) limit = UINT64_MAX;
    if (n > limit) {
      if (cfg.verbose)
        std::fprintf(stderr, "WARNING clustering %zu points to %zu centroids: sampling %llu points\n",
                     n, k, (unsigned long long)limit);
      keep = eb::host::Mt19937(cfg.seed ^ 0x9E3779B9u).permutation(n);
      keep.resize(limit);
      std::sort(keep.begin(), keep.end());
      sub.resize(limit * d);
      for (size_t i = 0; i < limit; i++)
        std::memcpy(&sub[i * d], data + (size_t)keep[i] * d, d * 4);
      x = sub.data();
      rows = limit;
      if (rows < k) throw Refused("need at least k = " + std::to_string(k) + " rows, got " + std::to_string(rows));
    }
  }

  eb_train_job job{};
  job.x = x;
  job.n = rows;
  job.d = d;
  job.k = k;
  job.nepochs = cfg.nepochs;
  job.batch_law = cfg.batch_law;
  job.spherical = cfg.spherical;
  job.batch_size = cfg.batch_size_set ? (int64_t)cfg.batch_size : 0;
  job.alpha0 = cfg.alpha0_set ? cfg.alpha0 : NAN;
  job.unused_threshold = cfg.tau_set ? cfg.unused_threshold : NAN;
  job.seed = cfg.seed;
  job.capture = cfg.capture_assignments;
  job.chunk = cfg.chunk_set ? (int64_t)cfg.assignment_chunk_size : 0;
  job.verbose = cfg.verbose;
  if (cfg.batch_size_set && cfg.batch_size == 0) throw Refused("batch_size must be positive");

  std::unique_ptr<EmeansModel> m(new EmeansModel);
  m->k = k;
  m->d = d;
  m->spherical = cfg.spherical;
  m->centroids.assign(k * d, 0.0f);
  std::vector<int32_t> lab(cfg.capture_assignments ? rows : 0);
  eb_train_out out{};
  out.centroids = m->centroids.data();
  out.labels = cfg.capture_assignments ? lab.data() : nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    eb_engine* e = engine_locked();
    engine_call(eb_train(e, &job, &out));
  }
  m->epochs = (size_t)out.n_epochs;
  if (out.n_epochs < 1) throw Refused("training ran no epoch");

  if (result_out) {
    std::unique_ptr<EmeansResult> r(new EmeansResult);
    r->arrays.emplace_back();
    r->arrays.back().name = "centroids";
    r->arrays.back().dtype = EMEANS_F32;
    r->arrays.back().f32 = m->centroids;
    if (cfg.capture_assignments) {
      std::vector<int32_t> all;
      if (keep.empty()) {
        all = std::move(lab);
      } else {
        all.assign(n, -1);
        for (size_t i = 0; i < keep.size(); i++) all[keep[i]] = lab[i];
      }
      r->arrays.emplace_back();
      r->arrays.back().name = "labels";
      r->arrays.back().dtype = EMEANS_I32;
      r->arrays.back().i32 = std::move(all);
    }
    // The last epoch's moving objective as a mean over its rows
    // (bindings/common/src/lib.rs:233-246).
    std::vector<size_t> epoch_rows;
    {
      eb::host::Recipe rc = eb::host::resolve_recipe(rows, k, d, cfg.nepochs, cfg.batch_law,
                                                     cfg.batch_size_set ? cfg.batch_size : 0,
                                                     cfg.alpha0_set ? cfg.alpha0 : NAN);
      epoch_rows = rc.epoch_rows;
    }
    const size_t ne = (size_t)out.n_epochs;
    if (epoch_rows.size() < ne || epoch_rows[ne - 1] == 0)
      throw Refused("no row count for the last epoch");
    const double objective = out.obj[ne - 1] / (double)epoch_rows[ne - 1];
    std::string exact = "null";
    if (cfg.exact_objective) {
      std::vector<uint32_t> l;
      std::vector<float> s;
      run_assign(data, n, d, m->centroids.data(), k, cfg.spherical ? EB_IP : EB_L2, l, s);
      exact = fmt_num(mean_objective(s, cfg.spherical));
    }
    std::string js = "{\"k\":" + std::to_string(k) + ",\"d\":" + std::to_string(d) +
                     ",\"objective\":" + fmt_num(objective) + ",\"exact_objective\":" + exact +
                     ",\"stats\":[";
    for (size_t ep = 0; ep < ne; ep++) {
      if (ep) js += ",";
      js += "{\"obj\":" + fmt_num(out.obj[ep]) + ",\"time\":" + fmt_num(out.epoch_time[ep]) +
            ",\"imbalance_factor\":" + fmt_num(out.imbalance[ep]) +
            ",\"nsplit\":" + std::to_string(out.nsplit[ep]) + "}";
    }
    js += "],\"backend\":\"b200\"}";
    r->json = js;
    *result_out = std::move(r);
  }
  if (model_out) *model_out = std::move(m);
}

const EmeansModel& need_model(const EmeansModel* m) {
  if (!m) throw BadArg("model is NULL");
  return *m;
}

}  // namespace

extern "C" {

uint32_t emeans_abi_version(void) { return EMEANS_ABI_VERSION; }

const char* emeans_version(void) { return "0.1.0"; }

const char* emeans_last_error(void) { return t_failed ? t_error.c_str() : nullptr; }

void emeans_string_free(char* s) { std::free(s); }

int32_t emeans_default_config(const char* kind, char** out_json) {
  return guard([&] {
    if (!out_json) throw BadArg("out_json is NULL");
    const std::string k(need_string(kind, "kind"));
    if (k == "auto" || k == "dedup") throw Refused("config kind \"" + k + "\" is not in this library (it has: train)");
    if (k != "train") throw Refused("unknown config kind \"" + k + "\" (one of train, auto, dedup)");
    *out_json = new_cstring(default_train_config());
  });
}

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
    *out_json = new_cstring(ok ? "[\"cuda\"]" : "[]");
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
    if (backend) check_backend(backend);
    std::vector<uint32_t> labels;
    std::vector<float> scores;
    run_assign(data, n, d, centroids, k, met, labels, scores);
    *out_result = assign_result(std::move(labels), std::move(scores)).release();
  });
}

int32_t emeans_train(const float* data, size_t n, size_t d, size_t k, const char* config_json,
                     EmeansResult** out_result) {
  return guard([&] {
    if (!out_result) throw BadArg("out_result is NULL");
    check_slice(data, mul(n, d), "data");
    std::unique_ptr<EmeansResult> r;
    train_model(data, n, d, k, config_json, nullptr, &r);
    *out_result = r.release();
  });
}

int32_t emeans_model_train(const float* data, size_t n, size_t d, size_t k,
                           const char* config_json, EmeansModel** out_model,
                           EmeansResult** out_result) {
  return guard([&] {
    if (!out_model) throw BadArg("out_model is NULL");
    check_slice(data, mul(n, d), "data");
    std::unique_ptr<EmeansModel> m;
    std::unique_ptr<EmeansResult> r;
    train_model(data, n, d, k, config_json, &m, out_result ? &r : nullptr);
    if (out_result) *out_result = r.release();
    *out_model = m.release();
  });
}

int32_t emeans_model_assign(const EmeansModel* m, const float* data, size_t n,
                            EmeansResult** out_result) {
  return guard([&] {
    if (!out_result) throw BadArg("out_result is NULL");
    const EmeansModel& md = need_model(m);
    check_slice(data, mul(n, md.d), "data");
    std::vector<uint32_t> labels;
    std::vector<float> scores;
    run_assign(data, n, md.d, md.centroids.data(), md.k, md.spherical ? EB_IP : EB_L2, labels,
               scores);
    *out_result = assign_result(std::move(labels), std::move(scores)).release();
  });
}

int32_t emeans_model_objective(const EmeansModel* m, const float* data, size_t n,
                               double* out_objective) {
  return guard([&] {
    if (!out_objective) throw BadArg("out_objective is NULL");
    const EmeansModel& md = need_model(m);
    check_slice(data, mul(n, md.d), "data");
    std::vector<uint32_t> labels;
    std::vector<float> scores;
    run_assign(data, n, md.d, md.centroids.data(), md.k, md.spherical ? EB_IP : EB_L2, labels,
               scores);
    *out_objective = mean_objective(scores, md.spherical);
  });
}

int32_t emeans_model_centroids(const EmeansModel* m, EmeansArray* out_array) {
  return guard([&] {
    const EmeansModel& md = need_model(m);
    if (!out_array) throw BadArg("out_array is NULL");
    *out_array = {md.centroids.empty() ? nullptr : md.centroids.data(), md.centroids.size(),
                  EMEANS_F32};
  });
}

int32_t emeans_model_info(const EmeansModel* m, char** out_json) {
  return guard([&] {
    if (!out_json) throw BadArg("out_json is NULL");
    const EmeansModel& md = need_model(m);
    *out_json = new_cstring(
        "{\"d\":" + std::to_string(md.d) + ",\"k\":" + std::to_string(md.k) + ",\"metric\":\"" +
        (md.spherical ? "inner_product" : "l2") + "\",\"spherical\":" +
        (md.spherical ? "true" : "false") + ",\"backend\":\"b200\",\"epochs\":" +
        std::to_string(md.epochs) + "}");
  });
}

void emeans_model_free(EmeansModel* m) { delete m; }

int32_t emeans_result_array(const EmeansResult* r, const char* name, EmeansArray* out_array) {
  return guard([&] {
    if (!r) throw BadArg("result is NULL");
    const std::string nm(need_string(name, "name"));
    const EmeansResult::Array* a = nullptr;
    for (const auto& x : r->arrays)
      if (x.name == nm) a = &x;
    if (!a) {
      std::string names;
      for (const auto& x : r->arrays) names += (names.empty() ? "" : ", ") + x.name;
      throw Refused("the result has no array \"" + nm + "\" (has: " + names + ")");
    }
    EmeansArray v{nullptr, 0, a->dtype};
    if (a->dtype == EMEANS_F32) v = {a->f32.data(), a->f32.size(), a->dtype};
    if (a->dtype == EMEANS_U32) v = {a->u32.data(), a->u32.size(), a->dtype};
    if (a->dtype == EMEANS_I32) v = {a->i32.data(), a->i32.size(), a->dtype};
    if (v.len == 0) v.data = nullptr;
    if (!out_array) throw BadArg("out_array is NULL");
    *out_array = v;
  });
}

const char* emeans_result_json(const EmeansResult* r) { return r ? r->json.c_str() : nullptr; }

void emeans_result_free(EmeansResult* r) { delete r; }

}  // extern "C"
