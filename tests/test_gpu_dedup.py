"""Near-duplicate grouping on the B200 (eb_dedup: the exact kNN self-join on
the engine, then the grouping stages of crates/emeans-cluster/src/dedup.rs)
against the oracle's pipeline (its FMA-chain self-join, then the Python
restatement of dedup_with_neighbors): every field equal, on a subsample of
the dedup config's shape (nested mixture, d = 768, 2% injected near-duplicates
at sigma 0.005, sim_threshold 0.97) and with bursts, times and priorities."""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from oracle import dedup as odedup

pytestmark = pytest.mark.gpu


def check(engine, x, d, cfg, created=None, burst=None, priority=None):
    got = engine.dedup(x, d, created, burst, priority, cfg)
    n = x.shape[0]
    kk = max(1, min(cfg.k, n - 1))
    ids, sims = oracle.topk(x.ravel(), x.ravel(), d, kk, exclude_self=True)
    want = odedup.dedup_with_neighbors(x, d, ids, sims, kk, created, burst, priority,
                                       cfg.sim_threshold, cfg.rep_threshold, cfg.max_gap_secs)
    for f in ("group_of", "representatives", "anchors", "sizes"):
        assert np.array_equal(getattr(got, f), want[f]), f
    assert np.array_equal(got.nn_sim.view(np.uint32), want["nn_sim"].view(np.uint32))
    assert got.linked_pairs == want["linked_pairs"]
    assert got.split_components == want["split_components"]
    return got


def test_dedup_config_shape_subsample(engine):
    from bench import gen_c5_rows

    n, d = 6000, 768
    x = gen_c5_rows(n, d, seed=9)
    r = check(engine, x, d, eb.DedupConfig(k=10, sim_threshold=0.97))
    assert r.n_groups() < n  # the injected near-duplicates group


def test_with_bursts_times_and_priorities(engine):
    rng = np.random.default_rng(4)
    n, d = 2500, 96
    x = rng.standard_normal((n, d)).astype(np.float32)
    x[2000:2200] = x[:200] + np.float32(0.05) * rng.standard_normal((200, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    created = rng.uniform(0, 600, n)
    created[rng.choice(n, 100, replace=False)] = np.nan
    burst = [None] * n
    for i in rng.choice(n, 300, replace=False):
        burst[i] = int(rng.integers(0, 40))
    priority = rng.integers(0, 2, n).astype(np.float32)
    cfg = eb.DedupConfig(k=8, sim_threshold=0.95, rep_threshold=0.9, max_gap_secs=300.0)
    check(engine, x, d, cfg, created, burst, priority)
