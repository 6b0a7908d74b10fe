"""CPU restatement of the reference's near-duplicate grouping (test
infrastructure: the checker for the engine's eb_dedup_with_neighbors / eb_dedup,
never on the product path).

Follows crates/emeans-cluster/src/dedup.rs:186-358 (``dedup_with_neighbors``)
step by step with Python sets and dicts, as the reference does with HashSet,
HashMap and BTreeMap:

- union-find with path halving where the lower root wins (dedup.rs:131-155);
- burst units from the first row of each burst id (dedup.rs:219-228);
- links: neighbour j of i with sim >= sim_threshold and the time rule
  (dedup.rs:208-216, 235-247), unordered pairs counted once in a set;
- components in the order of their lowest row, star cover by (more links,
  then lower id), a unit joins only when all its rows fit the anchor
  (dedup.rs:250-304);
- groups sorted by lowest member, representatives by priority, then mean
  f64 similarity in member order, then lowest id (dedup.rs:305-345).

``dot`` is the reference's ``a.iter().zip(b).map(|(p, q)| p * q).sum()``: f32
products rounded and added in column order (numpy's cumulative sum in f32 is
that sequential chain).
"""

from __future__ import annotations

import math

import numpy as np

NONE = 0xFFFFFFFF


def dot(a: np.ndarray, b: np.ndarray) -> np.float32:
    p = (a.astype(np.float32) * b.astype(np.float32)).astype(np.float32)
    return np.cumsum(p, dtype=np.float32)[-1] if p.size else np.float32(-0.0)


class _UnionFind:
    def __init__(self, n):
        self.p = list(range(n))

    def find(self, i):
        while self.p[i] != i:
            q = self.p[i]
            self.p[i] = self.p[q]
            i = q
        return i

    def union(self, a, b):
        ra, rb = self.find(a), self.find(b)
        if ra != rb:
            lo, hi = min(ra, rb), max(ra, rb)
            self.p[hi] = lo


def dedup_with_neighbors(x, d, ids, sims, kk, created=None, burst=None, priority=None,
                         sim_threshold=0.95, rep_threshold=None, max_gap_secs=None):
    """Returns dict(group_of, representatives, anchors, sizes, nn_sim,
    linked_pairs, split_components) like DedupResult. ``burst`` entries are
    None (no burst) or an int id; ``ids`` / ``sims`` are n x kk."""
    x = np.asarray(x, np.float32).reshape(-1, d)
    n = x.shape[0]
    ids = np.asarray(ids, np.uint32).reshape(n, kk)
    sims = np.asarray(sims, np.float32).reshape(n, kk)
    sim_t = np.float32(sim_threshold)
    rep_t = sim_t if rep_threshold is None else np.float32(rep_threshold)

    def time_ok(i, j):
        if max_gap_secs is None or created is None:
            return True
        ti, tj = created[i], created[j]
        if not (math.isfinite(ti) and math.isfinite(tj)):
            return True
        return abs(ti - tj) <= max_gap_secs

    unit = _UnionFind(n)
    if burst is not None:
        first = {}
        for i, b in enumerate(burst):
            if b is not None:
                f = first.setdefault(b, i)
                unit.union(f, i)
    comp = _UnionFind(n)
    for i in range(n):
        comp.union(unit.find(i), i)
    degree = [0] * n
    pairs = set()
    for i in range(n):
        for t in range(kk):
            j = int(ids[i, t])
            s = sims[i, t]
            if j == NONE or s < sim_t or not time_ok(i, j):
                continue
            comp.union(i, j)
            key = (min(i, j), max(i, j))
            if key not in pairs:
                pairs.add(key)
                degree[i] += 1
                degree[j] += 1

    members = {}
    for i in range(n):
        members.setdefault(comp.find(i), []).append(i)
    unit_of = [unit.find(i) for i in range(n)]

    groups = []  # (rows, anchor)
    split = 0
    for root in sorted(members):
        rows = members[root]
        if len(rows) == 1:
            groups.append((list(rows), rows[0]))
            continue
        units = {}
        for r in rows:
            units.setdefault(unit_of[r], []).append(r)
        order = sorted(rows, key=lambda r: (-degree[r], r))
        taken = set()
        before = len(groups)
        for c in order:
            cu = unit_of[c]
            if cu in taken:
                continue
            taken.add(cu)
            g = list(units[cu])
            rest = [u for u in sorted(units) if u not in taken]
            joins = [all(time_ok(r, c) and dot(x[r], x[c]) >= rep_t for r in units[u])
                     for u in rest]
            for u, jn in zip(rest, joins):
                if jn:
                    taken.add(u)
                    g.extend(units[u])
            g.sort()
            groups.append((g, c))
        if len(groups) - before > 1:
            split += 1
    groups.sort(key=lambda g: g[0][0])
    anchors = [g[1] for g in groups]
    groups = [g[0] for g in groups]

    reps = []
    for g in groups:
        if len(g) == 1:
            reps.append(g[0])
            continue
        best = (-math.inf, -math.inf, NONE)
        for a in g:
            total = 0.0
            for b in g:
                if b != a:
                    total += float(dot(x[a], x[b]))
            mean = total / (len(g) - 1)
            p = float(priority[a]) if priority is not None else 0.0
            if p > best[0] or (p == best[0] and mean > best[1]):
                best = (p, mean, a)
        reps.append(best[2])
    group_of = np.zeros(n, np.uint32)
    for gi, g in enumerate(groups):
        for r in g:
            group_of[r] = gi
    return dict(group_of=group_of, representatives=np.array(reps, np.uint32),
                anchors=np.array(anchors, np.uint32),
                sizes=np.array([len(g) for g in groups], np.uint32),
                nn_sim=sims[:, 0].copy(), linked_pairs=len(pairs), split_components=split)
