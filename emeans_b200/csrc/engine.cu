// The C ABI of the engine: engine and buffer management, argument checks that
// mirror the reference's (core/mod.rs:432-439 check_select, assign.rs:121-147
// check_shapes, crates/emeans-cuda/src/lib.rs:1129-1139), and dispatch of the
// layer-1 ops onto the engine's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_set>

#include "engine.h"

namespace {

thread_local std::string g_last_error;

template <class F>
int guard(F&& f) {
  try {
    f();
    g_last_error.clear();
    return EB_OK;
  } catch (const eb::Error& err) {
    g_last_error = err.what();
    return err.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host out of memory";
    return EB_ERROR;
  } catch (const std::exception& err) {
    g_last_error = std::string("internal: ") + err.what();
    return EB_INTERNAL;
  }
}

// Makes the engine's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(const eb_engine* e) {
    cudaGetDevice(&prev);
    if (prev != e->device) EB_CUDA(cudaSetDevice(e->device));
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void need(const void* p, const char* what) {
  eb::ensure(p != nullptr, std::string(what) + " is null");
}

void need_type(const eb_buf* b, int dtype, const char* what) {
  need(b, what);
  eb::ensure(b->dtype == dtype,
             std::string(what) + (dtype == EB_F32 ? " must be an f32 buffer" : " must be a u32 buffer"));
}

// An op wrote `b` on the device: drop the caches derived from its contents.
void touched(eb_engine* e, eb_buf* b) {
  if (!b) return;
  b->version++;
  eb::drop_f16(b);
  if (b->xnorm) {
    cudaFreeAsync(b->xnorm, e->stream);
    b->xnorm = nullptr;
  }
}

// check_select (core/mod.rs:432-439).
void check_select(size_t r0, size_t r1, const eb_buf* ids, size_t n) {
  eb::ensure(r0 <= r1, "bad row range");
  if (ids)
    eb::ensure(r1 <= ids->len, "row range past the ids");
  else
    eb::ensure(r1 <= n, "row range past the data");
}

}  // namespace

namespace eb {

eb_buf* new_buf(eb_engine* e, int dtype, size_t len) {
  auto* b = new eb_buf;
  b->dtype = dtype;
  b->len = len;
  b->owned = true;
  size_t bytes = std::max<size_t>(len * 4, 16);
  cudaError_t st = cudaMallocAsync(&b->ptr, bytes, e->stream);
  e->device_allocs++;
  if (st != cudaSuccess) {
    delete b;
    throw Error(EB_ERROR, std::string("device allocation of ") + std::to_string(bytes) +
                              " bytes failed: " + cudaGetErrorString(st));
  }
  EB_CUDA(cudaMemsetAsync(b->ptr, 0, bytes, e->stream));
  return b;
}

void free_buf(eb_engine* e, eb_buf* b) {
  if (!b) return;
  drop_f16(b);
  if (b->xnorm) cudaFreeAsync(b->xnorm, e->stream);
  if (b->owned && b->ptr) cudaFreeAsync(b->ptr, e->stream);
  delete b;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

void sync(eb_engine* e) {
  EB_CUDA(cudaMemcpyAsync(e->h_status, e->d_status, 4, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaStreamSynchronize(e->stream));
  uint32_t st = *e->h_status;
  if (st) {
    *e->h_status = 0;
    EB_CUDA(cudaMemsetAsync(e->d_status, 0, 4, e->stream));
    EB_CUDA(cudaStreamSynchronize(e->stream));
    if (st & ST_BAD_LABEL) throw Error(EB_INVALID_ARGUMENT, "label out of range");
    if (st & ST_BAD_ROW) throw Error(EB_INVALID_ARGUMENT, "row id out of range");
    if (st & ST_WAIT_TIMEOUT) throw Error(EB_ERROR, "device-side wait timed out");
    if (st & ST_BAD_STATE) throw Error(EB_INTERNAL, "device-side consistency check failed");
    throw Error(EB_INTERNAL, "device reported status " + std::to_string(st));
  }
}

}  // namespace eb

using eb::ensure;

extern "C" {

const char* eb_last_error(void) { return g_last_error.c_str(); }

const char* eb_version(void) { return "emeans_b200 0.1 (sm_100a)"; }

int eb_engine_create(int device, eb_engine** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    int count = 0;
    cudaError_t st = cudaGetDeviceCount(&count);
    if (st != cudaSuccess || count == 0)
      throw eb::Error(EB_ERROR, std::string("no CUDA device: ") + cudaGetErrorString(st));
    ensure(device >= 0 && device < count, "device index out of range");
    cudaDeviceProp prop{};
    EB_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw eb::Error(EB_ERROR, std::string("emeans_b200 needs an sm_100 (B200) device, got ") +
                                    prop.name + " sm_" + std::to_string(prop.major) +
                                    std::to_string(prop.minor));
    auto* e = new eb_engine;
    e->device = device;
    e->num_sms = prop.multiProcessorCount;
    int prev = -1;
    cudaGetDevice(&prev);
    try {
      EB_CUDA(cudaSetDevice(device));
      EB_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
      EB_CUDA(cudaMalloc(&e->d_status, 16));
      EB_CUDA(cudaMemset(e->d_status, 0, 16));
      EB_CUDA(cudaMallocHost(&e->h_status, 16));
      *e->h_status = 0;
      EB_CUDA(cudaMalloc(&e->d_counters, 4 * sizeof(unsigned long long)));
      EB_CUDA(cudaMemset(e->d_counters, 0, 4 * sizeof(unsigned long long)));
      const char* sc = getenv("EMEANS_B200_SCREEN");
      if (sc && (sc[0] == '0' || sc[0] == '1' || sc[0] == '2') && sc[1] == 0)
        e->screen_mode = sc[0] - '0';
    } catch (...) {
      if (prev >= 0) cudaSetDevice(prev);
      delete e;
      throw;
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = e;
  });
}

int eb_engine_destroy(eb_engine* e) {
  if (!e) return EB_OK;
  return guard([&] {
    DeviceGuard g(e);
    cudaStreamSynchronize(e->stream);
    eb::group_leave(e);
    for (auto& ev : e->screen_ev) {
      cudaEventDestroy(ev.first);
      cudaEventDestroy(ev.second);
    }
    if (e->bound) eb::free_buf(e, e->bound);
    for (auto& kv : e->scratch)
      if (kv.second.p) cudaFreeAsync(kv.second.p, e->stream);
    cudaStreamSynchronize(e->stream);
    if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
    if (e->down_stream) cudaStreamSynchronize(e->down_stream);
    for (cudaEvent_t v : e->stage_ev)
      if (v) cudaEventDestroy(v);
    for (auto& kv : e->pinned)
      if (kv.second.p) cudaFreeHost(kv.second.p);
    cudaFree(e->d_status);
    cudaFree(e->d_counters);
    cudaFreeHost(e->h_status);
    if (e->copy_stream) cudaStreamDestroy(e->copy_stream);
    if (e->down_stream) cudaStreamDestroy(e->down_stream);
    cudaStreamDestroy(e->stream);
    delete e;
  });
}

int eb_engine_name(eb_engine* e, char* buf, size_t cap) {
  return guard([&] {
    need(e, "engine");
    need(buf, "buf");
    std::string name = e->screen_mode ? "b200-exact" : "b200-exact-simt";
    ensure(cap > name.size(), "name buffer too small");
    std::memcpy(buf, name.c_str(), name.size() + 1);
  });
}

int eb_flush(eb_engine* e) {
  return guard([&] { need(e, "engine"); });
}

int eb_sync(eb_engine* e) {
  return guard([&] {
    need(e, "engine");
    DeviceGuard g(e);
    eb::sync(e);
  });
}

int eb_engine_stream(eb_engine* e, void** stream) {
  return guard([&] {
    need(e, "engine");
    need(stream, "stream");
    *stream = (void*)e->stream;
  });
}

int eb_get_stats(eb_engine* e, eb_stats* out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    DeviceGuard g(e);
    unsigned long long c[4];
    EB_CUDA(cudaMemcpyAsync(c, e->d_counters, sizeof(c), cudaMemcpyDeviceToHost, e->stream));
    eb::sync(e);
    *out = e->stats;
    out->fallback_rows = c[1];
    out->rescored_candidates = c[2];
  });
}

int eb_test_screen_dead_wait(eb_engine* e, int on) {
  return guard([&] {
    need(e, "engine");
    e->screen_dead_wait = on != 0;
  });
}

int eb_device_allocations(eb_engine* e, uint64_t* count) {
  return guard([&] {
    need(e, "engine");
    need(count, "count");
    *count = e->device_allocs;
  });
}

int eb_set_kernel_timing(eb_engine* e, int on) {
  return guard([&] {
    need(e, "engine");
    e->time_screen = on != 0;
  });
}

int eb_screen_timing(eb_engine* e, double* total_ms, uint64_t* launches, uint64_t* rows) {
  return guard([&] {
    need(e, "engine");
    need(total_ms, "total_ms");
    need(launches, "launches");
    need(rows, "rows");
    DeviceGuard g(e);
    eb::sync(e);
    double ms = 0.0;
    uint64_t r = 0;
    for (size_t u = 0; u < e->screen_ev_used; u++) {
      float t = 0.0f;
      EB_CUDA(cudaEventElapsedTime(&t, e->screen_ev[u].first, e->screen_ev[u].second));
      ms += t;
      r += e->screen_ev_rows[u];
    }
    *total_ms = ms;
    *launches = e->screen_ev_used;
    *rows = r;
    e->screen_ev_used = 0;
  });
}

int eb_set_screen_mode(eb_engine* e, int mode) {
  return guard([&] {
    need(e, "engine");
    ensure(mode >= 0 && mode <= 2, "screen mode must be 0 (off), 1 (auto) or 2 (always)");
    e->screen_mode = mode;
  });
}

int eb_buf_alloc(eb_engine* e, int dtype, size_t len, eb_buf** out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    ensure(dtype == EB_F32 || dtype == EB_U32, "unknown dtype");
    DeviceGuard g(e);
    *out = eb::new_buf(e, dtype, len);
  });
}

int eb_buf_wrap(eb_engine* e, int dtype, void* dev_ptr, size_t len, eb_buf** out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    ensure(dtype == EB_F32 || dtype == EB_U32, "unknown dtype");
    ensure(dev_ptr != nullptr || len == 0, "null device pointer");
    ensure(((uintptr_t)dev_ptr & 15) == 0, "device pointer must be 16-byte aligned");
    cudaPointerAttributes attr{};
    if (dev_ptr) {
      EB_CUDA(cudaPointerGetAttributes(&attr, dev_ptr));
      ensure(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
             "pointer is not device memory");
      ensure(attr.type == cudaMemoryTypeManaged || attr.device == e->device,
             "pointer is on another device");
    }
    auto* b = new eb_buf;
    b->ptr = dev_ptr;
    b->len = len;
    b->dtype = dtype;
    b->owned = false;
    *out = b;
  });
}

int eb_buf_free(eb_engine* e, eb_buf* b) {
  if (!b) return EB_OK;
  return guard([&] {
    need(e, "engine");
    DeviceGuard g(e);
    if (e->bound == b) e->bound = nullptr;
    eb::free_buf(e, b);
  });
}

size_t eb_buf_len(const eb_buf* b) { return b ? b->len : 0; }
void* eb_buf_ptr(const eb_buf* b) { return b ? b->ptr : nullptr; }

int eb_buf_write(eb_engine* e, eb_buf* b, size_t offset, const void* host, size_t len) {
  return guard([&] {
    need(e, "engine");
    need(b, "buffer");
    ensure(offset <= b->len && len <= b->len - offset, "write past the buffer");
    if (len == 0) return;
    need(host, "host");
    DeviceGuard g(e);
    eb::h2d(e, static_cast<char*>(b->ptr) + offset * 4, host, len * 4, e->stream);
    b->version++;
    eb::drop_f16(b);
    if (b->xnorm) {
      cudaFreeAsync(b->xnorm, e->stream);
      b->xnorm = nullptr;
    }
  });
}

int eb_buf_read(eb_engine* e, const eb_buf* b, size_t lo, size_t hi, void* host) {
  return guard([&] {
    need(e, "engine");
    need(b, "buffer");
    ensure(lo <= hi && hi <= b->len, "read past the buffer");
    DeviceGuard g(e);
    if (hi > lo) {
      need(host, "host");
      eb::d2h(e, host, static_cast<const char*>(b->ptr) + lo * 4, (hi - lo) * 4, e->stream);
    }
    eb::sync(e);
  });
}

int eb_buf_upload(eb_engine* e, int dtype, const void* host, size_t len, eb_buf** out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    ensure(dtype == EB_F32 || dtype == EB_U32, "unknown dtype");
    ensure(host != nullptr || len == 0, "host is null");
    DeviceGuard g(e);
    eb_buf* b = eb::new_buf(e, dtype, len);
    if (len) eb::h2d(e, b->ptr, host, len * 4, e->stream);
    *out = b;
  });
}

int eb_bind(eb_engine* e, const float* x, size_t n, size_t d, eb_buf** out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    ensure(d > 0, "d must be positive");
    ensure(x != nullptr || n == 0, "x is null");
    DeviceGuard g(e);
    eb_buf* b = eb::new_buf(e, EB_F32, n * d);
    if (n) eb::h2d(e, b->ptr, x, n * d * 4, e->stream);
    b->d = d;
    *out = b;
  });
}

int eb_top1(eb_engine* e, const eb_buf* x, size_t d, const eb_buf* ids, size_t r0, size_t r1,
            const eb_buf* centroids, const eb_buf* cnorm, size_t k, int metric, eb_buf* labels,
            eb_buf* scores) {
  return guard([&] {
    need(e, "engine");
    need_type(x, EB_F32, "x");
    ensure(d > 0, "d must be positive");
    ensure(metric == EB_L2 || metric == EB_IP, "unknown metric");
    if (ids) need_type(ids, EB_U32, "ids");
    need_type(centroids, EB_F32, "centroids");
    need_type(labels, EB_U32, "labels");
    need_type(scores, EB_F32, "scores");
    check_select(r0, r1, ids, x->len / d);
    ensure(r1 <= labels->len && r1 <= scores->len, "outputs too short");
    ensure(k > 0 && centroids->len == k * d, "centroids must be k x d");
    ensure(k <= 0xFFFFFFFFull, "k too large");
    if (metric == EB_L2) {
      ensure(cnorm != nullptr && cnorm->len >= k, "L2 needs centroid norms");
      need_type(cnorm, EB_F32, "cnorm");
    }
    if (r0 == r1) return;
    DeviceGuard g(e);
    touched(e, labels);
    touched(e, scores);
    eb::Top1Args a;
    a.x = static_cast<const float*>(x->ptr);
    a.n = x->len / d;
    a.d = d;
    a.ids = ids ? static_cast<const uint32_t*>(ids->ptr) : nullptr;
    a.r0 = r0;
    a.r1 = r1;
    a.c = static_cast<const float*>(centroids->ptr);
    a.cnorm = cnorm ? static_cast<const float*>(cnorm->ptr) : nullptr;
    a.k = k;
    a.metric = metric;
    a.labels = static_cast<uint32_t*>(labels->ptr);
    a.scores = static_cast<float*>(scores->ptr);
    a.xnorm = (x->xnorm && x->d == d) ? x->xnorm : nullptr;
    if (metric == EB_L2 && !a.xnorm && x->d == d) {
      // Bound data: keep its row norms (CPU float order) for every later call.
      float* xn = nullptr;
      EB_CUDA(cudaMallocAsync(&xn, std::max<size_t>(a.n, 1) * 4, e->stream));
      e->device_allocs++;
      eb::row_norms(e, a.x, a.n, d, xn);
      const_cast<eb_buf*>(x)->xnorm = xn;
      a.xnorm = xn;
    }
    eb::top1_dispatch(e, a, const_cast<eb_buf*>(x));
  });
}

int eb_topk(eb_engine* e, const float* queries, size_t m, const float* data, size_t n, size_t d,
            size_t kk, int exclude_self, uint32_t* ids, float* sims) {
  return guard([&] {
    need(e, "engine");
    ensure(d > 0, "d must be positive");
    ensure(kk >= 1 && kk <= 16, "kk must be 1..=16");
    ensure(n > 0, "no data rows");
    ensure(!exclude_self || m == n, "exclude_self needs queries == data");
    ensure(n <= 0xFFFFFFFEull, "too many data rows");
    if (m == 0) return;
    need(queries, "queries");
    need(data, "data");
    need(ids, "ids");
    need(sims, "sims");
    DeviceGuard g(e);
    eb::topk(e, queries, m, data, n, d, kk, exclude_self != 0, ids, sims);
  });
}

int eb_internal_scores(eb_engine* e, const float* x, size_t n, size_t d, const uint32_t* labels,
                       size_t k, eb_internal* out, uint64_t* sizes) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    ensure(d > 0, "x must be n x d");  // metrics.rs:116
    ensure(k <= 0x7FFFFFFFull, "k too large");
    if (n > 0) {
      need(x, "x");
      need(labels, "labels");
    }
    uint32_t bad = 0;
    for (size_t i = 0; i < n; i++) bad |= (uint32_t)(labels[i] >= k);
    ensure(bad == 0, "label out of range");  // metrics.rs:119-122
    DeviceGuard g(e);
    eb::internal_scores(e, x, n, d, labels, k, out, sizes);
  });
}

int eb_topk_group(eb_engine* e, const float* queries, size_t m, const float* shard,
                  size_t n_shard, size_t shard_offset, size_t n_total, size_t d, size_t kk,
                  int exclude_self, uint32_t* ids, float* sims) {
  return guard([&] {
    need(e, "engine");
    ensure(d > 0, "d must be positive");
    ensure(kk >= 1 && kk <= 16, "kk must be 1..=16");
    ensure(n_total > 0 && n_total <= 0xFFFFFFFEull, "n_total must be in 1 .. 2^32 - 2");
    ensure(shard_offset + n_shard <= n_total, "shard past the data");
    ensure(!exclude_self || m == n_total, "exclude_self needs queries == data");
    if (m == 0) return;
    need(queries, "queries");
    if (n_shard) need(shard, "shard");
    need(ids, "ids");
    need(sims, "sims");
    DeviceGuard g(e);
    eb::topk(e, queries, m, shard, n_shard, d, kk, exclude_self != 0, ids, sims, shard_offset,
             true);
  });
}

int eb_scatter_add(eb_engine* e, const eb_buf* x, size_t d, const eb_buf* ids, size_t r0,
                   size_t r1, const eb_buf* labels, size_t k, eb_buf* sums, eb_buf* counts,
                   eb_buf* acc) {
  return guard([&] {
    need(e, "engine");
    need_type(x, EB_F32, "x");
    ensure(d > 0, "d must be positive");
    if (ids) need_type(ids, EB_U32, "ids");
    need_type(labels, EB_U32, "labels");
    need_type(sums, EB_F32, "sums");
    need_type(counts, EB_U32, "counts");
    check_select(r0, r1, ids, x->len / d);
    ensure(sums->len == k * d && counts->len == k, "sums k x d, counts k");
    ensure(k > 0, "k must be positive");
    ensure(r1 <= labels->len, "labels too short");
    if (acc) {
      need_type(acc, EB_F32, "acc");
      ensure(acc->len == k * d, "acc must be k x d");
    }
    DeviceGuard g(e);
    touched(e, sums);
    touched(e, counts);
    touched(e, acc);
    eb::scatter_add(e, static_cast<const float*>(x->ptr), x->len / d, d,
                    ids ? static_cast<const uint32_t*>(ids->ptr) : nullptr, r0, r1,
                    static_cast<const uint32_t*>(labels->ptr), k, static_cast<float*>(sums->ptr),
                    static_cast<uint32_t*>(counts->ptr),
                    acc ? static_cast<float*>(acc->ptr) : nullptr);
  });
}

int eb_row_norms(eb_engine* e, const eb_buf* m, size_t rows, size_t d, eb_buf* out) {
  return guard([&] {
    need(e, "engine");
    need_type(m, EB_F32, "m");
    need_type(out, EB_F32, "out");
    ensure(m->len >= rows * d && out->len >= rows, "shapes");
    DeviceGuard g(e);
    touched(e, out);
    eb::row_norms(e, static_cast<const float*>(m->ptr), rows, d, static_cast<float*>(out->ptr));
  });
}

int eb_normalize_rows(eb_engine* e, const eb_buf* src, size_t rows, size_t d, eb_buf* dst) {
  return guard([&] {
    need(e, "engine");
    need_type(src, EB_F32, "src");
    need_type(dst, EB_F32, "dst");
    ensure(src->len >= rows * d && dst->len >= rows * d, "shapes");
    DeviceGuard g(e);
    touched(e, dst);
    eb::normalize_rows(e, static_cast<const float*>(src->ptr), rows, d,
                       static_cast<float*>(dst->ptr));
  });
}

int eb_split(eb_engine* e, eb_buf* positions, eb_buf* usage, const uint32_t* pairs, size_t npairs,
             size_t d) {
  return guard([&] {
    need(e, "engine");
    need_type(positions, EB_F32, "positions");
    need_type(usage, EB_F32, "usage");
    size_t k = usage->len;
    ensure(positions->len == k * d, "positions must be k x d");
    if (npairs == 0) return;
    need(pairs, "pairs");
    std::unordered_set<uint32_t> seen;
    for (size_t i = 0; i < 2 * npairs; i++) {
      ensure(pairs[i] < k, "split ids out of range");
      ensure(seen.insert(pairs[i]).second, "split pairs must not share ids");
    }
    DeviceGuard g(e);
    touched(e, positions);
    touched(e, usage);
    uint32_t* dp = e->scratch_get<uint32_t>("split_pairs", 2 * npairs);
    EB_CUDA(cudaMemcpyAsync(dp, pairs, 2 * npairs * 4, cudaMemcpyHostToDevice, e->stream));
    eb::split(e, static_cast<float*>(positions->ptr), static_cast<float*>(usage->ptr), dp, npairs,
              d);
  });
}

int eb_ema_update(eb_engine* e, eb_buf* positions, eb_buf* usage, const eb_buf* sums,
                  const eb_buf* counts, size_t k, size_t d, float alpha, float decay,
                  int replace) {
  return guard([&] {
    need(e, "engine");
    need_type(positions, EB_F32, "positions");
    need_type(usage, EB_F32, "usage");
    need_type(sums, EB_F32, "sums");
    need_type(counts, EB_U32, "counts");
    ensure(positions->len == k * d && usage->len == k && sums->len == k * d && counts->len == k,
           "shapes");
    DeviceGuard g(e);
    touched(e, positions);
    touched(e, usage);
    eb::ema_update(e, static_cast<float*>(positions->ptr), static_cast<float*>(usage->ptr),
                   static_cast<const float*>(sums->ptr), static_cast<const uint32_t*>(counts->ptr),
                   k, d, alpha, decay, replace != 0);
  });
}

int eb_bind_data(eb_engine* e, const float* data, size_t n, size_t d) {
  return guard([&] {
    need(e, "engine");
    ensure(d > 0, "d must be positive");
    DeviceGuard g(e);
    if (e->bound) {
      eb::free_buf(e, e->bound);
      e->bound = nullptr;
    }
    eb_buf* b = nullptr;
    int rc = eb_bind(e, data, n, d, &b);
    if (rc != EB_OK) throw eb::Error(rc, g_last_error);
    e->bound = b;
    e->bound_host = data;
    e->bound_n = n;
  });
}

int eb_unbind_data(eb_engine* e) {
  return guard([&] {
    need(e, "engine");
    DeviceGuard g(e);
    if (e->bound) eb::free_buf(e, e->bound);
    e->bound = nullptr;
    e->bound_host = nullptr;
    e->bound_n = 0;
  });
}

int eb_assign(eb_engine* e, const float* rows, size_t n, size_t d, const uint32_t* ids, size_t m,
              const float* centroids, size_t k, int metric, uint32_t* labels, float* scores) {
  return guard([&] {
    need(e, "engine");
    // check_shapes (assign.rs:121-147).
    ensure(d > 0, "d must be positive");
    ensure(k > 0 && centroids != nullptr, "centroids must be k x d");
    ensure(k <= 0xFFFFFFFFull, "k too large");
    ensure(metric == EB_L2 || metric == EB_IP, "unknown metric");
    if (ids) {
      for (size_t i = 0; i < m; i++) ensure(ids[i] < n, "row id out of range");
    } else {
      ensure(m == n, "dense rows: m must equal n");
    }
    if (m == 0) return;
    need(rows, "rows");
    need(labels, "labels");
    need(scores, "scores");
    DeviceGuard g(e);
    float* c = e->scratch_get<float>("as_c", k * d);
    eb::h2d(e, c, centroids, k * d * 4, e->stream);
    float* cn = nullptr;
    if (metric == EB_L2) {
      cn = e->scratch_get<float>("as_cn", k);
      eb::row_norms(e, c, k, d, cn);
    }
    uint32_t* lab = e->scratch_get<uint32_t>("as_lab", m);
    float* sco = e->scratch_get<float>("as_sco", m);
    eb_buf cb, cnb, lb, sb;
    cb.ptr = c; cb.len = k * d; cb.dtype = EB_F32;
    cnb.ptr = cn; cnb.len = k; cnb.dtype = EB_F32;
    lb.ptr = lab; lb.len = m; lb.dtype = EB_U32;
    sb.ptr = sco; sb.len = m; sb.dtype = EB_F32;
    int rc;
    if (ids && e->bound && e->bound_host == rows && e->bound_n == n && e->bound->d == d) {
      // Rows::Indexed on the bound data: only the ids travel (core/mod.rs:276-298).
      uint32_t* di = e->scratch_get<uint32_t>("as_ids", m);
      EB_CUDA(cudaMemcpyAsync(di, ids, m * 4, cudaMemcpyHostToDevice, e->stream));
      eb_buf ib;
      ib.ptr = di; ib.len = m; ib.dtype = EB_U32;
      rc = eb_top1(e, e->bound, d, &ib, 0, m, &cb, metric == EB_L2 ? &cnb : nullptr, k, metric,
                   &lb, &sb);
    } else if (ids) {
      // Indexed rows gathered on the host (core/mod.rs:299-325).
      float* xd = e->scratch_get<float>("as_x", m * d);
      std::vector<float> gbuf(m * d);
      for (size_t i = 0; i < m; i++)
        std::memcpy(&gbuf[i * d], rows + (size_t)ids[i] * d, d * 4);
      eb::h2d(e, xd, gbuf.data(), m * d * 4, e->stream);
      eb_buf xb;
      xb.ptr = xd; xb.len = m * d; xb.dtype = EB_F32;
      rc = eb_top1(e, &xb, d, nullptr, 0, m, &cb, metric == EB_L2 ? &cnb : nullptr, k, metric,
                   &lb, &sb);
    } else if (e->bound && e->bound_host == rows && e->bound_n == n && e->bound->d == d) {
      // Dense rows that are the bound data set (the host pointer and shape the
      // binding is served by, as for indexed rows): read in place with the
      // binding's norms and screen copy, so that every fit of a sweep over
      // one bound set assigns without uploading it again.
      rc = eb_top1(e, e->bound, d, nullptr, 0, m, &cb, metric == EB_L2 ? &cnb : nullptr, k,
                   metric, &lb, &sb);
    } else {
      // Dense rows: copied in slices on the copy stream, each slice's top-1
      // queued on the engine's stream behind its own copy, so that the copy
      // of slice j + 1 overlaps the top-1 of slice j. The last slice is
      // small (16,384 rows when there are at least 65,536), so that little
      // compute remains once the last copy has landed; with pinned output
      // buffers each slice's labels and scores go back as soon as they are
      // ready. The centroids' screen copy is made once, by the first slice
      // that takes the screen.
      float* xd = e->scratch_get<float>("as_x", m * d);
      if (!e->copy_stream) EB_CUDA(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking));
      std::vector<size_t> cut{0};
      if (m >= 65536) {
        const size_t body = m - 16384, third = (body + 2) / 3;
        for (size_t r = third; r < body; r += third) cut.push_back(r);
        cut.push_back(body);
      } else {
        const size_t slice = std::max<size_t>(16384, (m + 3) / 4);
        for (size_t r = slice; r < m; r += slice) cut.push_back(r);
      }
      cut.push_back(m);
      const bool early_out = eb::host_pinned(labels) && eb::host_pinned(scores);
      cudaEvent_t ready;
      EB_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
      EB_CUDA(cudaEventRecord(ready, e->stream));  // earlier work on the staging buffer
      EB_CUDA(cudaStreamWaitEvent(e->copy_stream, ready, 0));
      EB_CUDA(cudaEventDestroy(ready));
      bool converted = false;
      for (size_t j = 0; j + 1 < cut.size(); j++) {
        const size_t r0 = cut[j], r1 = cut[j + 1];
        if (r1 == r0) continue;
        eb::h2d(e, xd + r0 * d, rows + r0 * d, (r1 - r0) * d * 4, e->copy_stream);
        cudaEvent_t landed;
        EB_CUDA(cudaEventCreateWithFlags(&landed, cudaEventDisableTiming));
        EB_CUDA(cudaEventRecord(landed, e->copy_stream));
        EB_CUDA(cudaStreamWaitEvent(e->stream, landed, 0));
        EB_CUDA(cudaEventDestroy(landed));
        eb::Top1Args a;
        a.x = xd;
        a.n = m;
        a.d = d;
        a.ids = nullptr;
        a.r0 = r0;
        a.r1 = r1;
        a.c = c;
        a.cnorm = cn;
        a.k = k;
        a.metric = metric;
        a.labels = lab;
        a.scores = sco;
        a.xnorm = nullptr;
        a.centroids_ready = converted;
        const bool screened = eb::top1_screen_supported(e, a);
        eb::top1_dispatch(e, a, nullptr);
        converted = converted || screened;
        if (early_out) {
          EB_CUDA(cudaMemcpyAsync(labels + r0, lab + r0, (r1 - r0) * 4, cudaMemcpyDeviceToHost,
                                  e->stream));
          EB_CUDA(cudaMemcpyAsync(scores + r0, sco + r0, (r1 - r0) * 4, cudaMemcpyDeviceToHost,
                                  e->stream));
        }
      }
      if (early_out) {
        eb::sync(e);
        return;
      }
      rc = EB_OK;
    }
    if (rc != EB_OK) throw eb::Error(rc, g_last_error);
    eb::d2h(e, labels, lab, m * 4, e->stream);
    eb::d2h(e, scores, sco, m * 4, e->stream);
    eb::sync(e);
  });
}

}  // extern "C"
