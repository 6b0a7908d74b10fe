"""Near-duplicate grouping (dedup::dedup_with_neighbors, the host stages of
crates/emeans-cluster/src/dedup.rs:186-358) in the engine library, on CPU.

The neighbour lists come from the oracle's exact self-join (the engine's
eb_topk returns the same bits on the GPU, tests/test_gpu_topk.py); the C++
stages must return exactly what the Python restatement in oracle/dedup.py
returns (groups, representatives, anchors, sizes, nearest similarities, link
and split counts). The reference's own dedup tests
(crates/emeans-cluster/tests/dedup.rs:112-302) are restated with inputs of
the same construction: bursts recovered exactly, chains cut into stars of
bounded diameter, the time-gap rule, burst ids, priorities, and a burst that
joins a star only when every row fits.
"""

import math

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from oracle import dedup as odedup


def unit_rows(n, d, seed):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def neighbours(x, d, k):
    n = x.shape[0]
    kk = max(1, min(k, n - 1))
    if n == 1:
        return np.full(1, 0xFFFFFFFF, np.uint32), np.full(1, -np.inf, np.float32), 1
    ids, sims = oracle.topk(x.ravel(), x.ravel(), d, kk, exclude_self=True)
    return ids, sims, kk


def run_both(x, d, cfg=eb.DedupConfig(), created=None, burst=None, priority=None):
    ids, sims, kk = neighbours(x, d, cfg.k)
    got = eb.dedup_with_neighbors(x, d, ids, sims, kk, created, burst, priority, cfg)
    want = odedup.dedup_with_neighbors(x, d, ids, sims, kk, created, burst, priority,
                                       cfg.sim_threshold, cfg.rep_threshold, cfg.max_gap_secs)
    for f in ("group_of", "representatives", "anchors", "sizes"):
        assert np.array_equal(getattr(got, f), want[f]), f
    assert np.array_equal(got.nn_sim.view(np.uint32), want["nn_sim"].view(np.uint32))
    assert got.linked_pairs == want["linked_pairs"]
    assert got.split_components == want["split_components"]
    return got


def with_bursts(base, n_bursts, sizes, sigma, seed):
    """Base rows plus near-copies: n_bursts rows each copied 1..5 more times
    with noise sigma / sqrt(d) per column, renormalised; truth = the group of
    every row (copies share their original's group)."""
    rng = np.random.default_rng(seed)
    n, d = base.shape
    rows, truth = [base], list(range(n))
    for b in rng.choice(n, n_bursts, replace=False):
        for _ in range(rng.integers(sizes[0], sizes[1])):
            v = base[b] + sigma / math.sqrt(d) * rng.standard_normal(d)
            rows.append((v / np.linalg.norm(v)).astype(np.float32)[None])
            truth.append(int(b))
    return np.concatenate(rows).astype(np.float32), np.array(truth)


def test_matches_the_restatement_on_random_inputs():
    rng = np.random.default_rng(3)
    for case in range(6):
        n, d = int(rng.integers(40, 260)), int(rng.integers(8, 40))
        base = unit_rows(n, d, 10 + case)
        x, _ = with_bursts(base, n // 5, (1, 5), 0.15, case)
        m = x.shape[0]
        created = rng.uniform(0, 100, m) if case % 2 else None
        if created is not None:
            created[rng.choice(m, m // 10, replace=False)] = np.nan
        burst = [None] * m
        if case >= 3:
            for i in rng.choice(m, m // 8, replace=False):
                burst[i] = int(rng.integers(0, 6))
        priority = rng.integers(0, 3, m).astype(np.float32) if case % 3 == 0 else None
        cfg = eb.DedupConfig(k=int(rng.integers(1, 12)), sim_threshold=float(rng.uniform(0.6, 0.97)),
                             rep_threshold=None if case < 4 else 0.9,
                             max_gap_secs=30.0 if case % 2 else None)
        run_both(x, d, cfg, created, burst if case >= 3 else None, priority)


def test_recovers_injected_bursts():
    """dedup.rs tests:112-142: separated base rows plus near-copy bursts; the
    groups are exactly the bursts, every representative is in its group, and
    expand / gather follow the groups."""
    d = 128
    base = unit_rows(800, d, 21)
    x, truth = with_bursts(base, 40, (1, 6), 0.143, 5)
    r = run_both(x, d)
    assert r.n_groups() == 800
    # Same partition as the truth (the groups are numbered by lowest row,
    # and every burst's original is its lowest row).
    assert np.array_equal(r.group_of, np.unique(truth, return_inverse=True)[1])
    for g, rep in enumerate(r.representatives):
        assert r.group_of[rep] == g
    labels = np.arange(r.n_groups()) * 10
    assert np.array_equal(r.expand(labels), r.group_of * 10)
    assert r.gather(x, d).shape == (r.n_groups(), d)


def test_cuts_chains():
    """dedup.rs tests:144-182: a random walk whose steps have cosine ~0.976
    is cut into stars; any two members of a group are within twice the
    threshold angle."""
    d = 256
    rng = np.random.default_rng(8)
    x = [unit_rows(1, d, 1)[0]]
    for _ in range(1, 40):
        z = rng.standard_normal(d)
        z /= np.linalg.norm(z)
        v = x[-1] + 0.22 * z
        x.append((v / np.linalg.norm(v)).astype(np.float32))
    x = np.array(x, np.float32)
    assert float(odedup.dot(x[0], x[39])) < 0.8
    cfg = eb.DedupConfig()
    r = run_both(x, d, cfg)
    assert r.n_groups() > 1 and r.split_components >= 1
    t = cfg.sim_threshold
    for g in range(r.n_groups()):
        m = np.flatnonzero(r.group_of == g)
        for a in m:
            for b in m:
                assert float(odedup.dot(x[a], x[b])) >= 2 * t * t - 1 - 1e-4


def test_time_gap_bursts_and_priority():
    """dedup.rs tests:184-246."""
    d = 64
    x = unit_rows(4, d, 77)
    c = x[0] + 0.001
    x = np.vstack([x, (c / np.linalg.norm(c))[None]]).astype(np.float32)
    t = np.array([0.0, 10.0, 20.0, 30.0, 86_400.0])
    cfg = eb.DedupConfig()
    r = run_both(x, d, cfg)
    assert r.group_of[0] == r.group_of[4] and r.n_groups() == 4
    gap = eb.DedupConfig(max_gap_secs=60.0)
    r = run_both(x, d, gap, created=t)
    assert r.group_of[0] != r.group_of[4]
    t_nan = t.copy()
    t_nan[4] = np.nan
    r = run_both(x, d, gap, created=t_nan)
    assert r.group_of[0] == r.group_of[4]
    r = run_both(x, d, cfg, burst=[None, 7, 7, None, None])
    assert r.group_of[1] == r.group_of[2] and r.n_groups() == 3
    for fav in (0, 4):
        p = np.zeros(5, np.float32)
        p[fav] = 1.0
        r = run_both(x, d, cfg, priority=p)
        assert r.representatives[r.group_of[0]] == fav


def crafted(d, parts):
    v = np.zeros(d, np.float32)
    for a, w in parts:
        v[a] = w
    return (v / np.linalg.norm(v)).astype(np.float32)


def test_a_burst_joins_a_star_only_when_every_row_fits():
    """dedup.rs tests:260-302."""
    d = 32
    x = [crafted(d, [(0, 1.0)])]
    for a in (1, 2, 3):
        x.append(crafted(d, [(0, 0.96), (a, 0.28)]))
    x.append(crafted(d, [(0, 0.96), (4, 0.28)]))  # b1 = row 4
    x.append(crafted(d, [(9, 1.0)]))              # b2 = row 5
    x = np.array(x, np.float32)
    burst = [None, None, None, None, 1, 1]
    cfg = eb.DedupConfig()
    r = run_both(x, d, cfg, burst=burst)
    assert r.group_of[4] == r.group_of[5]
    assert r.group_of[5] != r.group_of[0]
    assert r.anchors.size == r.n_groups() and r.anchors[r.group_of[0]] == 0
    for i in range(6):
        a = int(r.anchors[r.group_of[i]])
        assert r.group_of[a] == r.group_of[i]
        same = burst[i] is not None and burst[i] == burst[a]
        assert same or float(odedup.dot(x[i], x[a])) >= cfg.sim_threshold - 1e-6


def test_one_row_and_argument_errors():
    x = unit_rows(1, 8, 2)
    r = run_both(x, 8)
    assert r.n_groups() == 1 and r.representatives[0] == 0 and r.nn_sim[0] == -np.inf
    x = unit_rows(5, 8, 3)
    ids, sims, kk = neighbours(x, 8, 3)
    with pytest.raises(eb.EngineError, match="sim_threshold"):
        eb.dedup_with_neighbors(x, 8, ids, sims, kk, cfg=eb.DedupConfig(sim_threshold=1.5))
    with pytest.raises(eb.EngineError, match="NaN"):
        eb.dedup_with_neighbors(x, 8, ids, sims, kk, priority=[0, 1, np.nan, 0, 0])
    bad = ids.copy()
    bad[0] = 99
    with pytest.raises(eb.EngineError, match="past the rows"):
        eb.dedup_with_neighbors(x, 8, bad, sims, kk)


def test_matches_the_restatement_with_large_components():
    """Clustered rows (a few hundred per mean, unit norm) at a threshold that
    links most of a cluster: components of hundreds of rows, whose star covers
    and representatives the library computes on several host threads at once,
    whole and split into several stars; every field equal to the
    restatement's."""
    rng = np.random.default_rng(17)
    d, means, per = 24, 6, 250
    mu = rng.standard_normal((means, d)).astype(np.float32)
    x = np.repeat(mu, per, axis=0) + np.float32(0.12) * rng.standard_normal(
        (means * per, d)).astype(np.float32)
    x = (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)
    x = x[rng.permutation(x.shape[0])]
    got = run_both(x, d, eb.DedupConfig(k=10, sim_threshold=0.95))
    assert got.sizes.max() >= 50  # the case exercises large components
    # A stricter representative threshold splits the components' star covers.
    got = run_both(x, d, eb.DedupConfig(k=10, sim_threshold=0.95, rep_threshold=0.985))
    assert got.split_components >= 2 and got.sizes.max() >= 50
