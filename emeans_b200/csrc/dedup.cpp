// Near-duplicate groups over the exact kNN self-join: the host stages of
// crates/emeans-cluster/src/dedup.rs:186-358 (dedup_with_neighbors), with the
// self-join on the engine (eb_topk) in eb_dedup.
//
// 1. Burst units: rows with the same burst id are one unit (union-find,
//    lower root wins, so every root is its set's lowest row).
// 2. Links: i - j for each neighbour j of i with sim >= sim_threshold and, when
//    both rows have a finite timestamp and max_gap_secs is set, a time gap <=
//    max_gap_secs; components = units joined by links. Each unordered pair is
//    counted once for the link degrees (the first row that reports it).
// 3. Star cover of each component: rows by (more links, then lower id); the
//    first row whose unit is not taken anchors a group with its unit, and
//    every other untaken unit joins when all its rows pass the time rule and
//    have dot >= rep_threshold with the anchor.
// 4. Groups ordered by their lowest row; the representative is the member
//    with the highest priority, then the highest mean f64 similarity to the
//    other members, then the lowest id.
// Dots are the reference's `a.iter().zip(b).map(|(p, q)| p * q).sum()`:
// rounded products added in column order (no contraction: the library is
// built with -ffp-contract=off), so every threshold test sees the same bits.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <exception>
#include <map>
#include <mutex>
#include <system_error>
#include <thread>
#include <unordered_map>
#include <vector>

#include "engine.h"

namespace eb {
namespace {

struct UnionFind {
  std::vector<uint32_t> p;
  explicit UnionFind(size_t n) : p(n) {
    for (size_t i = 0; i < n; i++) p[i] = (uint32_t)i;
  }
  uint32_t find(uint32_t i) {
    while (p[i] != i) {
      const uint32_t q = p[i];
      p[i] = p[q];  // path halving
      i = q;
    }
    return i;
  }
  void unite(uint32_t a, uint32_t b) {
    const uint32_t ra = find(a), rb = find(b);
    if (ra != rb) p[std::max(ra, rb)] = std::min(ra, rb);  // lower root wins
  }
};

float dot(const float* a, const float* b, size_t d) {
  float s = -0.0f;
  for (size_t t = 0; t < d; t++) s += a[t] * b[t];
  return s;
}

// out[l] = dot(a, b[l], d) for l < 8, computed together: eight independent
// chains, each the same rounded products added in column order from -0 as
// dot's (no contraction), so each result has dot's bits.
void dots8(const float* a, const float* const* b, size_t d, float* out) {
  float s0 = -0.0f, s1 = -0.0f, s2 = -0.0f, s3 = -0.0f;
  float s4 = -0.0f, s5 = -0.0f, s6 = -0.0f, s7 = -0.0f;
  const float *b0 = b[0], *b1 = b[1], *b2 = b[2], *b3 = b[3];
  const float *b4 = b[4], *b5 = b[5], *b6 = b[6], *b7 = b[7];
  for (size_t t = 0; t < d; t++) {
    const float v = a[t];
    s0 += v * b0[t];
    s1 += v * b1[t];
    s2 += v * b2[t];
    s3 += v * b3[t];
    s4 += v * b4[t];
    s5 += v * b5[t];
    s6 += v * b6[t];
    s7 += v * b7[t];
  }
  out[0] = s0;
  out[1] = s1;
  out[2] = s2;
  out[3] = s3;
  out[4] = s4;
  out[5] = s5;
  out[6] = s6;
  out[7] = s7;
}

// dot(a, rows[i]) for every i, eight at a time (the last group padded with a).
void dots_many(const float* a, const std::vector<const float*>& rows, size_t d, float* out) {
  const float* b[8];
  float o[8];
  for (size_t i0 = 0; i0 < rows.size(); i0 += 8) {
    const size_t m = std::min<size_t>(8, rows.size() - i0);
    for (size_t l = 0; l < 8; l++) b[l] = l < m ? rows[i0 + l] : a;
    dots8(a, b, d, o);
    for (size_t l = 0; l < m; l++) out[i0 + l] = o[l];
  }
}

// f(i) for i in [0, count) on the host's threads, items handed out one at a
// time (their costs differ by orders of magnitude). The first exception
// thrown by f is rethrown once every thread has stopped.
template <class F>
void parallel_for(size_t count, F&& f) {
  if (count == 0) return;
  const size_t hw = std::max<unsigned>(1u, std::thread::hardware_concurrency());
  const size_t nt = std::min<size_t>(std::min<size_t>(hw, 64), count);
  std::atomic<size_t> next{0};
  std::exception_ptr err;
  std::mutex mu;
  auto work = [&] {
    for (size_t i = next++; i < count; i = next++) {
      try {
        f(i);
      } catch (...) {
        std::lock_guard<std::mutex> lock(mu);
        if (!err) err = std::current_exception();
        next = count;
      }
    }
  };
  std::vector<std::thread> ts;
  // A thread the system refuses leaves its share to the threads that started.
  try {
    for (size_t t = 1; t < nt; t++) ts.emplace_back(work);
  } catch (const std::system_error&) {
  }
  work();
  for (auto& t : ts) t.join();
  if (err) std::rethrow_exception(err);
}

}  // namespace

void dedup_with_neighbors(const float* x, size_t n, size_t d, const uint32_t* ids,
                          const float* sims, size_t kk, const double* created,
                          const uint32_t* burst, const float* priority,
                          const eb_dedup_config* cfg, eb_dedup_out* out) {
  ensure(d > 0, "d must be positive");
  ensure(n == 0 || (x && ids && sims), "x, ids and sims are required");
  ensure(kk > 0, "kk must be positive");
  ensure(n < 0xFFFFFFFFull, "n must be below 2^32 - 1");
  ensure(cfg && out && out->group_of && out->representatives && out->anchors && out->sizes &&
             out->nn_sim,
         "config and every output array are required");
  const float sim_t = cfg->sim_threshold;
  ensure(sim_t >= -1.0f && sim_t <= 1.0f, "sim_threshold must be in [-1, 1]");
  const float rep_t = std::isnan(cfg->rep_threshold) ? sim_t : cfg->rep_threshold;
  const bool gap_rule = !std::isnan(cfg->max_gap_secs) && created != nullptr;
  const double gap = cfg->max_gap_secs;
  if (priority)
    for (size_t i = 0; i < n; i++) ensure(!std::isnan(priority[i]), "priority must not be NaN");
  auto time_ok = [&](size_t i, size_t j) {
    if (!gap_rule || !std::isfinite(created[i]) || !std::isfinite(created[j])) return true;
    return std::fabs(created[i] - created[j]) <= gap;
  };
  auto row = [&](size_t i) { return x + i * d; };
  auto passes = [&](size_t i, uint32_t j, float s) {
    return j != 0xFFFFFFFFu && !(s < sim_t) && time_ok(i, j);
  };
  for (size_t i = 0; i < n * kk; i++)
    ensure(ids[i] == 0xFFFFFFFFu || ids[i] < n, "a neighbour id is past the rows");

  // Burst units, then components of units and links.
  UnionFind unit(n);
  if (burst) {
    std::unordered_map<uint32_t, uint32_t> first;
    for (size_t i = 0; i < n; i++) {
      if (burst[i] == 0xFFFFFFFFu) continue;
      auto it = first.emplace(burst[i], (uint32_t)i).first;
      unit.unite(it->second, (uint32_t)i);
    }
  }
  UnionFind comp(n);
  for (size_t i = 0; i < n; i++) comp.unite(unit.find((uint32_t)i), (uint32_t)i);
  std::vector<uint32_t> degree(n, 0);
  uint64_t linked = 0;
  for (size_t i = 0; i < n; i++) {
    for (size_t t = 0; t < kk; t++) {
      const uint32_t j = ids[i * kk + t];
      if (!passes(i, j, sims[i * kk + t])) continue;
      comp.unite((uint32_t)i, j);
      // The pair is new unless a row before this one reported it: an earlier
      // entry of this row's list, or row j < i listing i with a passing link.
      bool seen = false;
      for (size_t u = 0; u < t && !seen; u++)
        seen = ids[i * kk + u] == j && passes(i, j, sims[i * kk + u]);
      if (!seen && j < i)
        for (size_t u = 0; u < kk && !seen; u++)
          seen = ids[(size_t)j * kk + u] == (uint32_t)i && passes(j, (uint32_t)i, sims[(size_t)j * kk + u]);
      if (!seen) {
        linked++;
        degree[i]++;
        degree[j]++;
      }
    }
  }

  // Members of each component in row order; components by their lowest row
  // (every root is its component's lowest row).
  std::vector<uint32_t> root(n), unit_of(n);
  for (size_t i = 0; i < n; i++) {
    root[i] = comp.find((uint32_t)i);
    unit_of[i] = unit.find((uint32_t)i);
  }
  std::vector<uint32_t> start(n + 1, 0), members(n);
  for (size_t i = 0; i < n; i++) start[root[i] + 1]++;
  for (size_t i = 0; i < n; i++) start[i + 1] += start[i];
  {
    std::vector<uint32_t> fill(start.begin(), start.end() - 1);
    for (size_t i = 0; i < n; i++) members[fill[root[i]]++] = (uint32_t)i;
  }

  struct Group {
    std::vector<uint32_t> rows;
    uint32_t anchor;
  };
  // The star cover of one component (its members in row order at
  // members[b, e)), appended to gs.
  auto cover = [&](uint32_t b, uint32_t e, std::vector<Group>& gs) {
    // Units of the component, by unit root (their rows in row order).
    std::map<uint32_t, std::vector<uint32_t>> units;
    for (uint32_t q = b; q < e; q++) units[unit_of[members[q]]].push_back(members[q]);
    std::vector<uint32_t> order(members.begin() + b, members.begin() + e);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t p, uint32_t q) {
      return degree[p] != degree[q] ? degree[p] > degree[q] : p < q;
    });
    std::map<uint32_t, bool> taken;
    for (auto& u : units) taken[u.first] = false;
    for (uint32_t a : order) {
      const uint32_t au = unit_of[a];
      if (taken[au]) continue;
      taken[au] = true;
      std::vector<uint32_t> g = units[au];
      // Each untaken unit joins when every one of its rows fits the anchor
      // (time rule, and dot >= rep_threshold); the rows' dots with the anchor
      // are computed eight at a time.
      std::vector<const float*> cand;
      for (auto& u : units)
        if (!taken[u.first])
          for (uint32_t r : u.second) cand.push_back(row(r));
      std::vector<float> dv(cand.size());
      dots_many(row(a), cand, d, dv.data());
      std::vector<uint32_t> joins;
      size_t ci = 0;
      for (auto& u : units) {
        if (taken[u.first]) continue;
        bool all = true;
        for (uint32_t r : u.second) {
          const float v = dv[ci++];  // every row's dot, in the order computed
          all = all && time_ok(r, a) && v >= rep_t;
        }
        if (all) joins.push_back(u.first);
      }
      for (uint32_t u : joins) {
        taken[u] = true;
        g.insert(g.end(), units[u].begin(), units[u].end());
      }
      std::sort(g.begin(), g.end());
      gs.push_back({std::move(g), a});
    }
  };
  // Components of two or more rows are covered on all host threads at once
  // (each on its own: the dots of a large component dominate the host
  // stages), their groups kept per component and then taken in component
  // order, as one thread would produce them.
  std::vector<uint32_t> multi;
  for (size_t c = 0; c < n; c++)
    if (start[c + 1] - start[c] > 1) multi.push_back((uint32_t)c);
  std::vector<std::vector<Group>> covered(multi.size());
  parallel_for(multi.size(), [&](size_t q) {
    cover(start[multi[q]], start[multi[q] + 1], covered[q]);
  });
  std::vector<Group> groups;
  uint64_t split_components = 0;
  for (size_t c = 0, q = 0; c < n; c++) {
    const uint32_t b = start[c], e = start[c + 1];
    if (b == e) continue;
    if (e - b == 1) {
      groups.push_back({{members[b]}, members[b]});
      continue;
    }
    std::vector<Group>& gs = covered[q++];
    if (gs.size() > 1) split_components++;
    for (Group& g : gs) groups.push_back(std::move(g));
  }
  std::stable_sort(groups.begin(), groups.end(),
                   [](const Group& p, const Group& q) { return p.rows[0] < q.rows[0]; });

  // Representatives: priority, then mean similarity to the other members
  // (f64, added in member order), then the lowest id; the groups on all host
  // threads at once (each group's sums in its own order).
  parallel_for(groups.size(), [&](size_t gi) {
    const std::vector<uint32_t>& g = groups[gi].rows;
    uint32_t rep = g[0];
    if (g.size() > 1) {
      float best_p = -INFINITY;
      double best_m = -INFINITY;
      rep = 0xFFFFFFFFu;
      std::vector<const float*> others;
      std::vector<float> dv(g.size());
      for (uint32_t a : g) {
        // The other members' dots with a (eight at a time), added in f64 in
        // member order.
        others.clear();
        for (uint32_t bb : g)
          if (bb != a) others.push_back(row(bb));
        dots_many(row(a), others, d, dv.data());
        double sum = -0.0;
        for (size_t i = 0; i < others.size(); i++) sum += (double)dv[i];
        const double mean = sum / (double)(g.size() - 1);
        const float p = priority ? priority[a] : 0.0f;
        if (p > best_p || (p == best_p && mean > best_m)) {
          best_p = p;
          best_m = mean;
          rep = a;
        }
      }
    }
    out->representatives[gi] = rep;
    out->anchors[gi] = groups[gi].anchor;
    out->sizes[gi] = (uint32_t)g.size();
    for (uint32_t r : g) out->group_of[r] = (uint32_t)gi;
  });
  for (size_t i = 0; i < n; i++) out->nn_sim[i] = sims[i * kk];
  out->n_groups = groups.size();
  out->linked_pairs = linked;
  out->split_components = split_components;
}

}  // namespace eb

extern "C" int eb_dedup_with_neighbors(const float* x, size_t n, size_t d, const uint32_t* ids,
                                       const float* sims, size_t kk, const double* created_unix,
                                       const uint32_t* burst, const float* priority,
                                       const eb_dedup_config* cfg, eb_dedup_out* out) {
  try {
    eb::dedup_with_neighbors(x, n, d, ids, sims, kk, created_unix, burst, priority, cfg, out);
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  } catch (const std::exception& err) {
    eb::set_last_error(std::string("internal: ") + err.what());
    return EB_INTERNAL;
  }
}

extern "C" int eb_dedup(eb_engine* e, const float* x, size_t n, size_t d,
                        const double* created_unix, const uint32_t* burst, const float* priority,
                        const eb_dedup_config* cfg, eb_dedup_out* out) {
  try {
    eb::ensure(e != nullptr && cfg != nullptr && out != nullptr, "engine, cfg and out are required");
    eb::ensure(d > 0, "d must be positive");
    eb::ensure(cfg->k >= 1 && cfg->k <= 16, "k must be in 1 ..= 16 on this engine");
    // k = min(cfg.k, n - 1), at least 1 (dedup.rs:172); one row has no neighbour.
    const size_t kk = std::max<size_t>(1, std::min<size_t>(cfg->k, n > 0 ? n - 1 : 0));
    std::vector<uint32_t> ids(n * kk, 0xFFFFFFFFu);
    std::vector<float> sims(n * kk, -INFINITY);
    if (n > 1) {
      const int rc = eb_topk(e, x, n, x, n, d, kk, 1, ids.data(), sims.data());
      if (rc != EB_OK) return rc;
    }
    eb::dedup_with_neighbors(x, n, d, ids.data(), sims.data(), kk, created_unix, burst, priority,
                             cfg, out);
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  } catch (const std::exception& err) {
    eb::set_last_error(std::string("internal: ") + err.what());
    return EB_INTERNAL;
  }
}
