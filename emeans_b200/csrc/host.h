// Host-side scalars of the training loop: numpy's legacy MT19937 streams
// (crates/emeans-core/src/rng.rs), the recipe (recipe.rs), the revival plan
// (core/mod.rs:339-370) and the closing means (core/mod.rs:404-429). These
// run on the CPU in the reference too; they decide the row order and the
// splits, so they reproduce the reference's arithmetic exactly.
#pragma once

#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <utility>
#include <vector>

namespace eb {
namespace host {

// numpy RandomState (rng.rs:13-103).
class Mt19937 {
 public:
  explicit Mt19937(uint32_t seed) {
    uint32_t s = seed;
    for (int i = 0; i < 624; i++) {
      st_[i] = s;
      s = 1812433253u * (s ^ (s >> 30)) + (uint32_t)(i + 1);
    }
    idx_ = 624;
  }
  uint32_t u32() {
    if (__builtin_expect(idx_ == 624, 0)) refill();
    return out_[idx_++];
  }
  // random_sample(): a 53-bit double in [0, 1) (rng.rs:63-67).
  double sample() {
    double a = (double)(u32() >> 5), b = (double)(u32() >> 6);
    return (a * 67108864.0 + b) / 9007199254740992.0;
  }
  // Uniform in [0, max] by masked rejection (rng.rs:70-92).
  uint64_t interval(uint64_t max) {
    if (max == 0) return 0;
    uint64_t mask = max;
    mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4;
    mask |= mask >> 8; mask |= mask >> 16; mask |= mask >> 32;
    if (max <= 0xffffffffull) {
      for (;;) {
        uint64_t v = u32() & mask;
        if (v <= max) return v;
      }
    }
    for (;;) {
      uint64_t hi = u32();
      uint64_t v = ((hi << 32) | u32()) & mask;
      if (v <= max) return v;
    }
  }
  // permutation(n) (rng.rs:95-102).
  // The same draws as swapping p[i] with p[interval(i)] for i = n-1 .. 1,
  // written without the rejection branch: each output either lands (swap,
  // next i) or is rejected (a swap of p[i] with itself, same i). The mask
  // only changes when i drops below a power of two, so it is computed once
  // per such range, which leaves a compare and a subtract between one draw's
  // i and the next.
  std::vector<uint32_t> permutation(size_t n) {
    std::vector<uint32_t> p(n);
    permutation_into(p.data(), n);
    return p;
  }
  void permutation_into(uint32_t* a, size_t n) {
    for (size_t i = 0; i < n; i++) a[i] = (uint32_t)i;
    if (n - 1 > 0xffffffffull) {
      for (size_t i = n; i-- > 1;) std::swap(a[i], a[(size_t)interval(i)]);
      return;
    }
    uint32_t i = n ? (uint32_t)(n - 1) : 0u;
    while (i > 0) {
      const uint32_t mask = 0xffffffffu >> __builtin_clz(i);
      for (const uint32_t low = mask >> 1; i > low;) {
        const uint32_t v = u32() & mask;
        const uint32_t take = v <= i;
        const uint32_t j = take ? v : i;
        const uint32_t t = a[i];
        a[i] = a[j];
        a[j] = t;
        i -= take;
      }
    }
  }

 private:
  static uint32_t twist(uint32_t a, uint32_t b, uint32_t c) {
    const uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
    return c ^ (y >> 1) ^ ((0u - (y & 1u)) & 0x9908b0dfu);
  }
  // The next 624 words of state, then all 624 outputs tempered at once (the
  // loops carry no modulo and the tempering vectorises).
  void refill() {
    int i = 0;
    for (; i < 227; i++) st_[i] = twist(st_[i], st_[i + 1], st_[i + 397]);
    for (; i < 623; i++) st_[i] = twist(st_[i], st_[i + 1], st_[i - 227]);
    st_[623] = twist(st_[623], st_[0], st_[396]);
    for (int j = 0; j < 624; j++) {
      uint32_t y = st_[j];
      y ^= y >> 11;
      y ^= (y << 7) & 0x9d2c5680u;
      y ^= (y << 15) & 0xefc60000u;
      out_[j] = y ^ (y >> 18);
    }
    idx_ = 0;
  }
  uint32_t st_[624];
  uint32_t out_[624];
  int idx_;
};

inline uint32_t epoch_seed(uint32_t seed, size_t epoch) {  // recipe.rs:246-248
  return (uint32_t)(((uint64_t)seed * 1000003ull + epoch) & 0xffffffffull);
}

struct Recipe {
  size_t batch_size = 1;
  double alpha0 = 1.0;
  std::vector<size_t> epoch_rows;
  size_t total_steps = 0;
};

inline size_t pow2_round(double v) {  // recipe.rs:172-183
  if (v <= 1.0) return 1;
  double lo = std::ldexp(1.0, (int)std::floor(std::log2(v)));
  return (size_t)(v / lo < (2.0 * lo) / v ? lo : 2.0 * lo);
}

// Recipe::resolve (recipe.rs:199-254); law 0 auto, 1 throughput, 2 quality.
inline Recipe resolve_recipe(size_t n, size_t k, size_t d, double nepochs, int law,
                             size_t given_batch, double given_alpha0) {
  Recipe r;
  if (law == 0) law = d <= 16 ? 2 : 1;
  size_t b;
  if (given_batch) {
    b = std::min(given_batch, n);
  } else {
    const double cb = law == 1 ? 0.035134 : 0.00439175;
    double raw = cb * std::pow((double)k, 0.134749) * std::pow((double)n, 0.876473) *
                 std::pow(nepochs, 0.813344);
    b = pow2_round(raw);
    b = law == 1 ? std::min(b, pow2_round((double)n / 2.0)) : std::min(b, n / 2);
    b = std::max<size_t>(std::min(b, n), 1);
  }
  r.batch_size = b;
  if (std::isnan(given_alpha0)) {
    double a = 0.8244 * std::pow((double)k, -0.4617) * std::pow((double)b, 0.9003) *
               std::pow((double)n, -0.4498) * std::pow(nepochs, -0.1057);
    r.alpha0 = std::min(std::max(a, 1e-4), 1.0);
  } else {
    r.alpha0 = given_alpha0;
  }
  double whole = std::floor(nepochs);
  size_t rem = (size_t)std::nearbyint((nepochs - whole) * (double)n);
  size_t w = (size_t)whole;
  if (w == 0) {
    r.epoch_rows.push_back(rem);
  } else {
    r.epoch_rows.assign(w - 1, n);
    if (rem) r.epoch_rows.push_back(rem);
    r.epoch_rows.push_back(n);
  }
  for (size_t rows : r.epoch_rows) r.total_steps += (rows + b - 1) / b;
  return r;
}

// Cosine-annealed EMA step (recipe.rs:251-255).
inline double scheduled_alpha(double alpha0, size_t step, size_t total) {
  double frac = (double)std::min(step, total) / (double)std::max<size_t>(total, 1);
  double cosine = 0.5 * (1.0 + std::cos(M_PI * frac));
  return alpha0 * (0.1 + (1.0 - 0.1) * cosine);
}

// numpy float32 pairwise summation (model.rs:970-1002).
inline float numpy_sum(const float* a, size_t n) {
  if (n < 8) {
    float s = 0.0f;
    for (size_t i = 0; i < n; i++) s = s + a[i];
    return s;
  }
  if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    size_t i = 8;
    for (; i < n - n % 8; i += 8)
      for (int j = 0; j < 8; j++) r[j] = r[j] + a[i + j];
    float s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) s = s + a[i];
    return s;
  }
  size_t h = n / 2;
  h -= h % 8;
  return numpy_sum(a, h) + numpy_sum(a + h, n - h);
}

// The random part of a revival plan: g[j] = log(-log(u_j)) for k uniforms
// u_j (floored at the smallest normal double), and the generator after
// drawing them. They depend only on the generator's state, so they can be
// drawn ahead, while the device runs the steps before the revival.
struct RevivalDraws {
  std::vector<double> g;
  Mt19937 after;
};
inline RevivalDraws revival_draws(Mt19937 rng, size_t k) {
  std::vector<double> g(k);
  for (auto& v : g) v = std::log(-std::log(std::max(rng.sample(), 2.2250738585072014e-308)));
  return {std::move(g), rng};
}

// plan_revival (core/mod.rs:339-370): (donor, dead) pairs, flattened. The
// uniforms are drawn only when there is something to split; `pre`, if given,
// holds them drawn ahead from rng's current state (rng then jumps to the state
// after them).
inline std::vector<uint32_t> plan_revival(const std::vector<float>& usage, double tau,
                                          Mt19937& rng, const RevivalDraws* pre = nullptr) {
  const size_t k = usage.size();
  std::vector<uint32_t> plan;
  float threshold = (numpy_sum(usage.data(), k) * (float)tau) / (float)k;
  size_t n_dead = 0, n_donor = 0;
  for (float u : usage) {
    bool dead = u < threshold;
    n_dead += dead;
    n_donor += !dead && u > 0.0f;
  }
  size_t nsplit = std::min(n_dead, n_donor);
  if (nsplit == 0) return plan;
  RevivalDraws own{{}, rng};
  if (!pre || pre->g.size() != k) {
    own = revival_draws(rng, k);
    pre = &own;
  }
  rng = pre->after;
  // Keys in IEEE total order (the reference's total_cmp) as unsigned
  // integers: the sign bit set flips every bit, else only the sign bit.
  struct Key {
    uint64_t key;
    uint32_t j;
  };
  std::vector<Key> keys;
  keys.reserve(n_donor);
  for (size_t j = 0; j < k; j++) {
    float u = usage[j];
    if (!(u < threshold) && u > 0.0f) {
      const double v = (double)std::log(u) - pre->g[j];
      uint64_t bits;
      std::memcpy(&bits, &v, 8);
      bits = (bits >> 63) ? ~bits : bits | 0x8000000000000000ull;
      keys.push_back({bits, (uint32_t)j});
    }
  }
  // Larger key first, then larger index: a strict order (indices differ), so
  // selecting the first nsplit and sorting them equals a stable sort's head.
  auto before = [](const Key& a, const Key& b) { return a.key != b.key ? a.key > b.key : a.j > b.j; };
  if (nsplit < keys.size()) std::nth_element(keys.begin(), keys.begin() + nsplit, keys.end(), before);
  std::sort(keys.begin(), keys.begin() + nsplit, before);
  plan.reserve(2 * nsplit);
  size_t t = 0;
  for (size_t i = 0; i < nsplit; i++) {
    while (!(usage[t] < threshold)) t++;
    plan.push_back(keys[i].j);
    plan.push_back((uint32_t)t++);
  }
  return plan;
}

// faiss normalize_into for one row (model.rs:954-967).
inline void normalize_row(float* r, size_t d) {
  float mx = 0.0f;
  for (size_t t = 0; t < d; t++) mx = std::fmax(mx, std::fabs(r[t]));
  float s = mx > 0.0f ? mx : 1.0f;
  for (size_t t = 0; t < d; t++) r[t] = r[t] / s;
  float ss = -0.0f;
  for (size_t t = 0; t < d; t++) ss = ss + r[t] * r[t];
  float nrm = std::sqrt(ss);
  s = nrm > 0.0f ? nrm : 1.0f;
  for (size_t t = 0; t < d; t++) r[t] = r[t] / s;
}

// closing_means (core/mod.rs:404-429).
inline void closing_means(const float* pos, const float* sums, const std::vector<double>& counts,
                          size_t k, size_t d, bool spherical, float* out) {
  std::memcpy(out, pos, k * d * sizeof(float));
  for (size_t j = 0; j < k; j++) {
    float* c = out + j * d;
    if (counts[j] > 0.0) {
      float nf = (float)counts[j];
      for (size_t t = 0; t < d; t++) c[t] = sums[j * d + t] / nf;
    }
    if (spherical) normalize_row(c, d);
  }
}

}  // namespace host
}  // namespace eb
