// CPU oracle for the emeans hot path. TEST INFRASTRUCTURE ONLY: the checker
// the CUDA engine is compared against, and the timed CPU baseline. The
// product library never links or calls this file.
//
// Restates the float order of the reference CPU path (crate emeans-core):
// every function cites the reference file:line it follows. Build with
// -ffp-contract=off so that only explicit std::fma / _mm256_fmadd_ps fuse.
#include "oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;
int fail(const std::string& m) {
  g_err = m;
  return 1;
}

// ---------------------------------------------------------------- MT19937
// numpy legacy RandomState (crates/emeans-core/src/rng.rs:13-103).
struct Mt {
  uint32_t mt[624];
  int pos;
  explicit Mt(uint32_t seed) {
    uint32_t s = seed;
    for (int i = 0; i < 624; i++) {
      mt[i] = s;
      s = 1812433253u * (s ^ (s >> 30)) + (uint32_t)(i + 1);
    }
    pos = 624;
  }
  void generate() {
    for (int i = 0; i < 624; i++) {
      uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
      uint32_t v = mt[(i + 397) % 624] ^ (y >> 1);
      if (y & 1u) v ^= 0x9908b0dfu;
      mt[i] = v;
    }
    pos = 0;
  }
  uint32_t next_u32() {
    if (pos == 624) generate();
    uint32_t y = mt[pos++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    return y ^ (y >> 18);
  }
  uint64_t next_u64() {
    uint64_t hi = next_u32();
    return (hi << 32) | next_u32();
  }
  // rng.rs:63-67
  double random_sample() {
    double a = (double)(next_u32() >> 5);
    double b = (double)(next_u32() >> 6);
    return (a * 67108864.0 + b) / 9007199254740992.0;
  }
  // rng.rs:70-92
  uint64_t random_interval(uint64_t max) {
    if (max == 0) return 0;
    uint64_t mask = max;
    for (int s : {1, 2, 4, 8, 16, 32}) mask |= mask >> s;
    if (max <= 0xffffffffull) {
      for (;;) {
        uint64_t v = (uint64_t)next_u32() & mask;
        if (v <= max) return v;
      }
    }
    for (;;) {
      uint64_t v = next_u64() & mask;
      if (v <= max) return v;
    }
  }
  // rng.rs:95-102
  void permutation(size_t n, uint32_t* out) {
    for (size_t i = 0; i < n; i++) out[i] = (uint32_t)i;
    for (size_t i = n; i-- > 1;) {
      size_t j = (size_t)random_interval(i);
      std::swap(out[i], out[j]);
    }
  }
};

// ---------------------------------------------------------------- recipe
// crates/emeans-core/src/recipe.rs
constexpr double kAlphaMinFactor = 0.1;
constexpr size_t kCheckUnusedEvery = 5;
constexpr float kInitUsage = 1.0f / 65536.0f;
constexpr double kSplitEpsilon = 1e-4;

size_t round_power_of_two(double value) {  // recipe.rs:172-183
  if (value <= 1.0) return 1;
  double low = std::ldexp(1.0, (int)std::floor(std::log2(value)));
  double high = 2.0 * low;
  return (size_t)(value / low < high / value ? low : high);
}

double step_law(size_t n, size_t k, double nepochs, size_t b) {  // recipe.rs:186-194
  double a = 0.8244 * std::pow((double)k, -0.4617) * std::pow((double)b, 0.9003) *
             std::pow((double)n, -0.4498) * std::pow(nepochs, -0.1057);
  return std::min(std::max(a, 1e-4), 1.0);
}

struct Recipe {
  size_t batch_size = 0;
  double alpha0 = 0;
  int resolved_law = 0;
  std::vector<size_t> epoch_rows;
  std::vector<size_t> epoch_steps;
  size_t total_steps = 0;
  size_t steps_per_pass = 0;
};

Recipe resolve(size_t n, size_t k, size_t d, double nepochs, int law, size_t batch_size,
               double alpha0) {  // recipe.rs:199-254
  Recipe r;
  if (law == ORC_LAW_AUTO) law = d <= 16 ? ORC_LAW_QUALITY : ORC_LAW_THROUGHPUT;
  size_t b;
  if (batch_size) {
    b = std::min(batch_size, n);
  } else {
    double c, bk, bn, bt;
    if (law == ORC_LAW_THROUGHPUT) {
      c = 0.035134; bk = 0.134749; bn = 0.876473; bt = 0.813344;
    } else {
      c = 0.00439175; bk = 0.134749; bn = 0.876473; bt = 0.813344;
    }
    double raw = c * std::pow((double)k, bk) * std::pow((double)n, bn) * std::pow(nepochs, bt);
    b = round_power_of_two(raw);
    if (law == ORC_LAW_THROUGHPUT)
      b = std::min(b, round_power_of_two((double)n / 2.0));
    else
      b = std::min(b, n / 2);
    b = std::max(std::min(b, n), (size_t)1);
    r.resolved_law = law;
  }
  r.batch_size = b;
  r.alpha0 = std::isnan(alpha0) ? step_law(n, k, nepochs, b) : alpha0;
  // recipe.rs:230-243
  double whole = std::floor(nepochs);
  size_t rem = (size_t)std::nearbyint((nepochs - whole) * (double)n);
  size_t w = (size_t)whole;
  if (w == 0) {
    r.epoch_rows.push_back(rem);
  } else {
    for (size_t i = 0; i + 1 < w; i++) r.epoch_rows.push_back(n);
    if (rem > 0) r.epoch_rows.push_back(rem);
    r.epoch_rows.push_back(n);
  }
  for (size_t rows : r.epoch_rows) {
    r.epoch_steps.push_back((rows + b - 1) / b);
    r.total_steps += r.epoch_steps.back();
  }
  r.steps_per_pass = (n + b - 1) / b;
  return r;
}

double scheduled_alpha(double alpha0, size_t step, size_t total) {  // recipe.rs:251-255
  double fraction = (double)std::min(step, total) / (double)std::max(total, (size_t)1);
  double cosine = 0.5 * (1.0 + std::cos(M_PI * fraction));
  return alpha0 * (kAlphaMinFactor + (1.0 - kAlphaMinFactor) * cosine);
}

uint32_t epoch_seed(uint32_t seed, size_t e) {  // recipe.rs:246-248
  return (uint32_t)(((uint64_t)seed * 1000003ull + (uint64_t)e) % (1ull << 32));
}

// ---------------------------------------------------------------- threads
void parallel_for(size_t tasks, int threads, const std::function<void(size_t)>& f) {
  if (threads <= 1 || tasks <= 1) {
    for (size_t t = 0; t < tasks; t++) f(t);
    return;
  }
  std::atomic<size_t> next{0};
  std::vector<std::thread> pool;
  int nt = (int)std::min<size_t>((size_t)threads, tasks);
  for (int i = 0; i < nt; i++)
    pool.emplace_back([&] {
      for (size_t t; (t = next.fetch_add(1)) < tasks;) f(t);
    });
  for (auto& th : pool) th.join();
}

// ---------------------------------------------------------------- norms
// Sequential sum of rounded squares, no FMA (assign.rs:150-155; Rust's
// `iter().map(|v| v * v).sum()`).
float sumsq(const float* r, size_t d) {
  float s = -0.0f;
  for (size_t t = 0; t < d; t++) s = s + r[t] * r[t];
  return s;
}

// faiss normalize_into for one row (core/cpu.rs:219-230, model.rs:954-967).
void normalize_row(float* r, size_t d) {
  float mx = 0.0f;
  for (size_t t = 0; t < d; t++) mx = std::fmax(mx, std::fabs(r[t]));
  float s = mx > 0.0f ? mx : 1.0f;
  for (size_t t = 0; t < d; t++) r[t] = r[t] / s;
  float nrm = std::sqrt(sumsq(r, d));
  s = nrm > 0.0f ? nrm : 1.0f;
  for (size_t t = 0; t < d; t++) r[t] = r[t] / s;
}

// ---------------------------------------------------------------- top-1
// The cpu-fused kernel's float order (assign/fused.rs:12-16,147-225):
// acc = 0; acc = fma(x_t, c_t, acc) for t = 0..d-1; IP: strict '>' scan from
// (-inf, 0); L2: key = cnorm_j - 2 acc (one rounding), strict '<' scan from
// (+inf, 0); score = max(sumsq(x) + key, 0) (assign.rs:423-502).
constexpr int MR = 6, NR = 16;

void pack_panels(const float* c, size_t k, size_t d, std::vector<float>& out) {
  size_t panels = (k + NR - 1) / NR;
  out.assign(panels * d * NR, 0.0f);
  for (size_t p = 0; p < panels; p++)
    for (int j = 0; j < NR && p * NR + j < k; j++) {
      const float* src = c + (p * NR + j) * d;
      for (size_t t = 0; t < d; t++) out[(p * d + t) * NR + j] = src[t];
    }
}

// dots[i][j] for MR rows (packed [d][MR]) x NR centroids (packed [d][NR]).
__attribute__((target("avx2,fma"))) void micro_avx2(const float* a, const float* b, size_t d,
                                                    float* out /* MR x NR */) {
  __m256 acc[MR][2];
  for (int i = 0; i < MR; i++) acc[i][0] = acc[i][1] = _mm256_setzero_ps();
  for (size_t t = 0; t < d; t++) {
    __m256 b0 = _mm256_loadu_ps(b + t * NR), b1 = _mm256_loadu_ps(b + t * NR + 8);
    for (int i = 0; i < MR; i++) {
      __m256 ai = _mm256_broadcast_ss(a + t * MR + i);
      acc[i][0] = _mm256_fmadd_ps(ai, b0, acc[i][0]);
      acc[i][1] = _mm256_fmadd_ps(ai, b1, acc[i][1]);
    }
  }
  for (int i = 0; i < MR; i++) {
    _mm256_storeu_ps(out + i * NR, acc[i][0]);
    _mm256_storeu_ps(out + i * NR + 8, acc[i][1]);
  }
}

void micro_portable(const float* a, const float* b, size_t d, float* out) {
  float acc[MR][NR] = {};
  for (size_t t = 0; t < d; t++)
    for (int i = 0; i < MR; i++)
      for (int j = 0; j < NR; j++) acc[i][j] = std::fma(a[t * MR + i], b[t * NR + j], acc[i][j]);
  std::memcpy(out, acc, sizeof(acc));
}

bool has_avx2() { return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"); }

void top1_rows(const float* x, size_t d, const uint32_t* ids, size_t r0, size_t r1,
               const std::vector<float>& packed, size_t k, int metric, const float* cnorm,
               uint32_t* labels, float* scores, int threads) {
  size_t m = r1 - r0;
  size_t tasks = (m + MR - 1) / MR;
  size_t panels = (k + NR - 1) / NR;
  bool avx = has_avx2();
  parallel_for(tasks, threads, [&](size_t task) {
    std::vector<float> a(d * MR, 0.0f);
    float dots[MR * NR];
    size_t p0 = r0 + task * MR;
    int nr = (int)std::min<size_t>(MR, r1 - p0);
    for (int i = 0; i < nr; i++) {
      size_t p = p0 + i;
      const float* row = x + (size_t)(ids ? ids[p] : p) * d;
      for (size_t t = 0; t < d; t++) a[t * MR + i] = row[t];
    }
    float best[MR];
    uint32_t bj[MR];
    for (int i = 0; i < MR; i++) {
      best[i] = metric == ORC_IP ? -INFINITY : INFINITY;
      bj[i] = 0;
    }
    for (size_t p = 0; p < panels; p++) {
      const float* b = packed.data() + p * d * NR;
      if (avx)
        micro_avx2(a.data(), b, d, dots);
      else
        micro_portable(a.data(), b, d, dots);
      int nc = (int)std::min<size_t>(NR, k - p * NR);
      for (int i = 0; i < nr; i++)
        for (int j = 0; j < nc; j++) {
          uint32_t col = (uint32_t)(p * NR + j);
          float v = dots[i * NR + j];
          if (metric == ORC_IP) {
            if (v > best[i]) { best[i] = v; bj[i] = col; }
          } else {
            float key = cnorm[col] - 2.0f * v;
            if (key < best[i]) { best[i] = key; bj[i] = col; }
          }
        }
    }
    for (int i = 0; i < nr; i++) {
      size_t p = p0 + i;
      labels[p] = bj[i];
      if (metric == ORC_IP) {
        scores[p] = best[i];
      } else {
        const float* row = x + (size_t)(ids ? ids[p] : p) * d;
        scores[p] = std::fmax(sumsq(row, d) + best[i], 0.0f);
      }
    }
  });
}

// numpy FLOAT_pairwise_sum (model.rs:970-1002).
float pairwise(const float* a, size_t n) {
  if (n < 8) {
    float res = 0.0f;
    for (size_t i = 0; i < n; i++) res = res + a[i];
    return res;
  } else if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    size_t i = 8;
    for (; i < n - n % 8; i += 8)
      for (int j = 0; j < 8; j++) r[j] = r[j] + a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) res = res + a[i];
    return res;
  }
  size_t n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise(a, n2) + pairwise(a + n2, n - n2);
}

// plan_revival (core/mod.rs:339-370).
std::vector<std::pair<uint32_t, uint32_t>> plan_revival(const float* usage, size_t k, double tau,
                                                        Mt& rng) {
  std::vector<std::pair<uint32_t, uint32_t>> plan;
  float total = pairwise(usage, k);
  float threshold = (total * (float)tau) / (float)k;
  std::vector<char> unused(k), donor(k);
  size_t n_unused = 0, n_donors = 0;
  for (size_t j = 0; j < k; j++) {
    unused[j] = usage[j] < threshold;
    donor[j] = !unused[j] && usage[j] > 0.0f;
    n_unused += unused[j];
    n_donors += donor[j];
  }
  size_t nsplit = std::min(n_unused, n_donors);
  if (nsplit == 0) return plan;
  std::vector<double> uni(k);
  for (size_t j = 0; j < k; j++) uni[j] = std::max(rng.random_sample(), 2.2250738585072014e-308);
  std::vector<std::pair<double, uint32_t>> keyed;
  for (size_t j = 0; j < k; j++)
    if (donor[j])
      keyed.push_back({(double)std::log(usage[j]) - std::log(-std::log(uni[j])), (uint32_t)j});
  // Descending key (total order; keys here are finite or -inf), ties: higher index first.
  std::stable_sort(keyed.begin(), keyed.end(), [](const auto& a, const auto& b) {
    if (a.first != b.first) return a.first > b.first;
    return a.second > b.second;
  });
  size_t t = 0;
  for (size_t i = 0; i < nsplit; i++) {
    while (!unused[t]) t++;
    plan.push_back({keyed[i].second, (uint32_t)t});
    t++;
  }
  return plan;
}

// apply_splits (core/mod.rs:374-399).
void apply_splits(float* pos, float* usage, size_t d, const uint32_t* pairs, size_t np) {
  float eps = (float)kSplitEpsilon;
  std::vector<float> donor(d), child(d);
  for (size_t q = 0; q < np; q++) {
    uint32_t s = pairs[2 * q], t = pairs[2 * q + 1];
    const float* c = pos + (size_t)s * d;
    bool same = true;
    for (size_t i = 0; i < d; i++) {
      float off = eps * (i % 2 == 0 ? 1.0f : -1.0f);
      donor[i] = c[i] * (1.0f - off);
      child[i] = c[i] * (1.0f + off);
      same = same && donor[i] == child[i];
    }
    if (same && d > 0) {
      float up = std::nextafter(child[0], INFINITY);
      child[0] = std::isfinite(up) ? up : std::nextafter(child[0], -INFINITY);
    }
    float half = usage[s] / 2.0f;
    usage[s] = half;
    std::memcpy(pos + (size_t)s * d, donor.data(), d * 4);
    usage[t] = half;
    std::memcpy(pos + (size_t)t * d, child.data(), d * 4);
  }
}

// ema_here (core/cpu.rs:389-432).
void ema(float* pos, float* usage, const float* sums, const uint32_t* counts, size_t k, size_t d,
         float a32, float decay, bool replace) {
  if (!replace)
    for (size_t j = 0; j < k; j++) usage[j] = usage[j] * decay;
  for (size_t j = 0; j < k; j++) {
    if (counts[j] == 0) continue;
    float count = (float)counts[j];
    float retained = replace ? 0.0f : usage[j];
    float step = a32 * count;
    float mass = retained + step;
    float weight = step / mass;
    float* c = pos + j * d;
    const float* s = sums + j * d;
    for (size_t t = 0; t < d; t++) {
      float mean = s[t] / count;
      c[t] = weight == 1.0f ? mean : c[t] + weight * (mean - c[t]);
    }
    usage[j] = mass;
  }
}

// scatter_rows (core/cpu.rs:233-252, 337-375): counts overwritten, sums[j] =
// rows with label j added in selection order from +0, acc += sums.
int scatter(const float* x, size_t d, const uint32_t* ids, size_t r0, size_t r1,
            const uint32_t* labels, size_t k, float* sums, uint32_t* counts, float* acc) {
  for (size_t p = r0; p < r1; p++)
    if (labels[p] >= k) return fail("label out of range");
  std::memset(counts, 0, k * 4);
  for (size_t i = 0; i < k * d; i++) sums[i] = 0.0f;
  for (size_t p = r0; p < r1; p++) {
    uint32_t l = labels[p];
    counts[l]++;
    const float* row = x + (size_t)(ids ? ids[p] : p) * d;
    float* s = sums + (size_t)l * d;
    for (size_t t = 0; t < d; t++) s[t] = s[t] + row[t];
  }
  if (acc)
    for (size_t i = 0; i < k * d; i++) acc[i] = acc[i] + sums[i];
  return 0;
}

// closing_means (core/mod.rs:404-429).
void closing(const float* pos, const float* sums, const double* counts, size_t k, size_t d,
             bool spherical, float* out) {
  std::memcpy(out, pos, k * d * 4);
  for (size_t j = 0; j < k; j++) {
    float* c = out + j * d;
    if (counts[j] > 0.0) {
      float nf = (float)counts[j];
      for (size_t t = 0; t < d; t++) c[t] = sums[j * d + t] / nf;
    }
    if (spherical) normalize_row(c, d);
  }
}

}  // namespace

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }

void orc_permutation(uint32_t seed, size_t n, uint32_t* out) { Mt(seed).permutation(n, out); }

void orc_random_sample(uint32_t seed, size_t count, double* out) {
  Mt r(seed);
  for (size_t i = 0; i < count; i++) out[i] = r.random_sample();
}

int orc_recipe(size_t n, size_t k, size_t d, double nepochs, int law, size_t batch_size,
               double alpha0, orc_recipe_t* out) {
  if (n == 0 || k == 0) return fail("n and k must be positive");
  Recipe r = resolve(n, k, d, nepochs, law, batch_size, alpha0);
  if (r.epoch_rows.size() > 64) return fail("too many epochs");
  out->batch_size = (int64_t)r.batch_size;
  out->alpha0 = r.alpha0;
  out->resolved_law = r.resolved_law;
  out->n_epochs = (int32_t)r.epoch_rows.size();
  out->steps_per_pass = (int64_t)r.steps_per_pass;
  out->total_steps = (int64_t)r.total_steps;
  for (size_t e = 0; e < r.epoch_rows.size(); e++) {
    out->epoch_rows[e] = (int64_t)r.epoch_rows[e];
    out->epoch_steps[e] = (int64_t)r.epoch_steps[e];
  }
  return 0;
}

double orc_scheduled_alpha(double alpha0, size_t step, size_t total) {
  return scheduled_alpha(alpha0, step, total);
}

double orc_unused_threshold(double given, size_t d) {  // recipe.rs:258-268
  if (std::isnan(given)) return d <= 2 ? 0.0 : 0.1;
  return given;
}

uint32_t orc_epoch_seed(uint32_t seed, size_t epoch) { return epoch_seed(seed, epoch); }

void orc_row_norms(const float* m, size_t rows, size_t d, float* out) {
  for (size_t i = 0; i < rows; i++) out[i] = sumsq(m + i * d, d);
}

void orc_normalize_rows(const float* src, size_t rows, size_t d, float* dst) {
  if (dst != src) std::memcpy(dst, src, rows * d * 4);
  for (size_t i = 0; i < rows; i++) normalize_row(dst + i * d, d);
}

int orc_top1(const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0, size_t r1,
             const float* c, size_t k, int metric, uint32_t* labels, float* scores,
             int threads) {
  if (d == 0 || k == 0) return fail("d and k must be positive");
  if (r0 > r1) return fail("bad row range");
  if (!ids && r1 > n) return fail("row range past the data");
  if (ids)
    for (size_t p = r0; p < r1; p++)
      if (ids[p] >= n) return fail("row id out of range");
  std::vector<float> packed, cn;
  pack_panels(c, k, d, packed);
  if (metric == ORC_L2) {
    cn.resize(k);
    orc_row_norms(c, k, d, cn.data());
  }
  top1_rows(x, d, ids, r0, r1, packed, k, metric, cn.data(), labels, scores, threads);
  return 0;
}

int orc_scatter_add(const float* x, size_t n, size_t d, const uint32_t* ids, size_t r0,
                    size_t r1, const uint32_t* labels, size_t k, float* sums,
                    uint32_t* counts, float* acc) {
  if (r0 > r1 || (!ids && r1 > n)) return fail("bad row range");
  return scatter(x, d, ids, r0, r1, labels, k, sums, counts, acc);
}

void orc_ema_update(float* pos, float* usage, const float* sums, const uint32_t* counts,
                    size_t k, size_t d, float alpha, float decay, int replace) {
  ema(pos, usage, sums, counts, k, d, alpha, decay, replace != 0);
}

void orc_split(float* pos, float* usage, size_t k, size_t d, const uint32_t* pairs,
               size_t npairs) {
  (void)k;
  apply_splits(pos, usage, d, pairs, npairs);
}

float orc_numpy_sum_f32(const float* a, size_t n) { return pairwise(a, n); }

void* orc_rng_new(uint32_t seed) { return new Mt(seed); }
void orc_rng_free(void* rng) { delete static_cast<Mt*>(rng); }

size_t orc_plan_revival(const float* usage, size_t k, double tau, void* rng, uint32_t* pairs_out) {
  auto plan = plan_revival(usage, k, tau, *static_cast<Mt*>(rng));
  for (size_t i = 0; i < plan.size(); i++) {
    pairs_out[2 * i] = plan[i].first;
    pairs_out[2 * i + 1] = plan[i].second;
  }
  return plan.size();
}

void orc_closing_means(const float* pos, const float* sums, const double* counts, size_t k,
                       size_t d, int spherical, float* out) {
  closing(pos, sums, counts, k, d, spherical != 0, out);
}

namespace {
// Query i's own column is self0 + i when exclude_self.
int topk_impl(const float* q, size_t m, const float* data, size_t n, size_t d, size_t kk,
              int exclude_self, size_t self0, uint32_t* ids, float* sims, int threads) {
  std::vector<float> packed;
  pack_panels(data, n, d, packed);
  size_t panels = (n + NR - 1) / NR;
  bool avx = has_avx2();
  size_t tasks = (m + MR - 1) / MR;
  parallel_for(tasks, threads, [&](size_t task) {
    std::vector<float> a(d * MR, 0.0f);
    float dots[MR * NR];
    size_t i0 = task * MR;
    int nr = (int)std::min<size_t>(MR, m - i0);
    for (int i = 0; i < nr; i++)
      for (size_t t = 0; t < d; t++) a[t * MR + i] = q[(i0 + i) * d + t];
    // Per query: best kk as (score desc, id asc); slot kk-1 is the worst.
    std::vector<float> bs(MR * kk, -INFINITY);
    std::vector<uint32_t> bi(MR * kk, UINT32_MAX);
    for (size_t p = 0; p < panels; p++) {
      const float* b = packed.data() + p * d * NR;
      if (avx)
        micro_avx2(a.data(), b, d, dots);
      else
        micro_portable(a.data(), b, d, dots);
      int nc = (int)std::min<size_t>(NR, n - p * NR);
      for (int i = 0; i < nr; i++) {
        float* s = bs.data() + i * kk;
        uint32_t* id = bi.data() + i * kk;
        for (int j = 0; j < nc; j++) {
          uint32_t col = (uint32_t)(p * NR + j);
          if (exclude_self && col == self0 + i0 + i) continue;
          float v = dots[i * NR + j];
          // Columns arrive in increasing id, so an equal score never displaces
          // (knn.rs:86: strict '>'); NaN and -inf never enter.
          if (!(v > s[kk - 1])) continue;
          size_t w = kk - 1;
          while (w > 0 && v > s[w - 1]) {
            s[w] = s[w - 1];
            id[w] = id[w - 1];
            w--;
          }
          // Insert after equal scores (which carry lower ids).
          s[w] = v;
          id[w] = col;
        }
      }
    }
    for (int i = 0; i < nr; i++)
      for (size_t t = 0; t < kk; t++) {
        ids[(i0 + i) * kk + t] = bi[i * kk + t];
        sims[(i0 + i) * kk + t] = bi[i * kk + t] == UINT32_MAX ? -INFINITY : bs[i * kk + t];
      }
  });
  return 0;
}
}  // namespace

int orc_topk(const float* q, size_t m, const float* data, size_t n, size_t d, size_t kk,
             int exclude_self, uint32_t* ids, float* sims, int threads) {
  if (d == 0 || kk == 0) return fail("d and kk must be positive");
  if (exclude_self && m != n) return fail("exclude_self needs queries == data");
  return topk_impl(q, m, data, n, d, kk, exclude_self, 0, ids, sims, threads);
}

// knn_self restricted to the queries data[q0 .. q0 + m): the self-join's
// results for those rows (each skips its own column q0 + i).
int orc_topk_self_rows(const float* data, size_t n, size_t d, size_t q0, size_t m, size_t kk,
                       uint32_t* ids, float* sims, int threads) {
  if (d == 0 || kk == 0) return fail("d and kk must be positive");
  if (q0 + m > n) return fail("query rows past the data");
  return topk_impl(data + q0 * d, m, data, n, d, kk, 1, q0, ids, sims, threads);
}

// The device loop (core/train.rs:60-303) on the oracle's ops.
int orc_train(const float* x, size_t n, size_t d, size_t k, const orc_train_cfg* cfg,
              const float* init, const float* state_pos, const float* state_usage,
              orc_train_out* out) {
  if (d == 0 || k == 0) return fail("d and k must be positive");
  if (n < k) return fail("need at least k rows");
  bool spherical = cfg->spherical != 0;
  int threads = cfg->threads > 0 ? cfg->threads : 1;
  double tau = orc_unused_threshold(cfg->unused_threshold, d);
  Recipe r = resolve(n, k, d, cfg->nepochs, cfg->batch_law, (size_t)cfg->batch_size,
                     cfg->alpha0);
  if (r.epoch_rows.size() > 64) return fail("too many epochs");
  for (size_t rows : r.epoch_rows)
    if (rows == 0) return fail("nepochs gives an empty epoch");
  // Start state (model.rs:306-317, 772-811).
  std::vector<float> pos(k * d), usage(k, kInitUsage);
  if (state_pos) {
    std::memcpy(pos.data(), state_pos, k * d * 4);
    std::memcpy(usage.data(), state_usage, k * 4);
  } else {
    if (init) {
      std::memcpy(pos.data(), init, k * d * 4);
    } else if (n == k) {
      std::memcpy(pos.data(), x, k * d * 4);
    } else {
      std::vector<uint32_t> perm(n);
      Mt(cfg->seed).permutation(n, perm.data());
      for (size_t j = 0; j < k; j++) std::memcpy(&pos[j * d], x + (size_t)perm[j] * d, d * 4);
    }
    if (spherical)
      for (size_t j = 0; j < k; j++) normalize_row(&pos[j * d], d);
  }
  size_t bsz = r.batch_size;
  size_t chunk = cfg->chunk > 0 ? (size_t)cfg->chunk : 65536;
  size_t n_epochs = r.epoch_rows.size();
  std::vector<uint32_t> order(n), labels_ep(n);
  std::vector<float> scores_ep(n), readout(spherical ? k * d : k), sums(k * d), pass(k * d, 0.0f);
  std::vector<uint32_t> counts(k);
  std::vector<double> pass_counts(k, 0.0);
  Mt split_rng(cfg->seed);
  size_t n_splits = 0, step = 0;
  std::vector<float> packed;
  std::vector<uint32_t> plan_buf(2 * k);
  if (out->labels)
    for (size_t i = 0; i < n; i++) out->labels[i] = -1;
  for (size_t epoch = 0; epoch < n_epochs; epoch++) {
    size_t rows = r.epoch_rows[epoch];
    Mt(epoch_seed(cfg->seed, epoch)).permutation(n, order.data());
    bool last = epoch + 1 == n_epochs;
    size_t splits_before = n_splits;
    for (size_t b = 0; b < rows; b += bsz) {
      size_t e = std::min(b + bsz, rows);
      if (spherical) {
        orc_normalize_rows(pos.data(), k, d, readout.data());
      } else {
        orc_row_norms(pos.data(), k, d, readout.data());
      }
      const float* cents = spherical ? readout.data() : pos.data();
      pack_panels(cents, k, d, packed);
      for (size_t c0 = b; c0 < e; c0 += chunk) {
        size_t c1 = std::min(c0 + chunk, e);
        top1_rows(x, d, order.data(), c0, c1, packed, k, spherical ? ORC_IP : ORC_L2,
                  spherical ? nullptr : readout.data(), labels_ep.data(), scores_ep.data(),
                  threads);
      }
      if (scatter(x, d, order.data(), b, e, labels_ep.data(), k, sums.data(), counts.data(),
                  last ? pass.data() : nullptr))
        return 1;
      double alpha = scheduled_alpha(r.alpha0, step, r.total_steps);
      ema(pos.data(), usage.data(), sums.data(), counts.data(), k, d, (float)alpha,
          (float)(1.0 - alpha), alpha == 1.0);
      if ((step + 1) % kCheckUnusedEvery == 0) {
        auto plan = plan_revival(usage.data(), k, tau, split_rng);
        if (!plan.empty()) {
          for (size_t i = 0; i < plan.size(); i++) {
            plan_buf[2 * i] = plan[i].first;
            plan_buf[2 * i + 1] = plan[i].second;
          }
          apply_splits(pos.data(), usage.data(), d, plan_buf.data(), plan.size());
          n_splits += plan.size();
        }
      }
      step++;
    }
    // Epoch statistics (train.rs:224-279).
    double obj_epoch = 0.0;
    for (size_t b = 0; b < rows; b += bsz) {
      size_t e = std::min(b + bsz, rows);
      double obj_batch = 0.0;
      for (size_t c0 = b; c0 < e; c0 += chunk) {
        size_t c1 = std::min(c0 + chunk, e);
        double obj = 0.0;
        if (spherical) {
          obj += 2.0 * (double)(c1 - c0);
          for (size_t i = c0; i < c1; i++) obj += (double)(-2.0f * scores_ep[i]);
        } else {
          for (size_t i = c0; i < c1; i++) obj += (double)scores_ep[i];
        }
        obj_batch += obj;
      }
      obj_epoch += obj_batch;
    }
    std::vector<uint64_t> hist(k, 0);
    for (size_t i = 0; i < rows; i++) hist[labels_ep[i]]++;
    double count_square = 0.0;
    for (size_t j = 0; j < k; j++) count_square += (double)hist[j] * (double)hist[j];
    out->obj[epoch] = obj_epoch;
    out->imbalance[epoch] = (double)k * count_square / ((double)rows * (double)rows);
    out->nsplit[epoch] = (int64_t)(n_splits - splits_before);
    if (last) {
      for (size_t j = 0; j < k; j++) pass_counts[j] = (double)hist[j];
      if (out->labels)
        for (size_t i = 0; i < rows; i++) out->labels[order[i]] = (int32_t)labels_ep[i];
    }
  }
  closing(pos.data(), pass.data(), pass_counts.data(), k, d, spherical, out->centroids);
  if (out->positions) std::memcpy(out->positions, pos.data(), k * d * 4);
  if (out->usage) std::memcpy(out->usage, usage.data(), k * 4);
  out->n_epochs = (int32_t)n_epochs;
  out->n_splits = (int64_t)n_splits;
  out->batch_size = (int64_t)bsz;
  out->alpha0 = r.alpha0;
  return 0;
}

}  // extern "C"
