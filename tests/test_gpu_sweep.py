"""The ``auto::fit`` sweep path on the engine (crates/emeans-cluster/src/auto.rs:
343-375): many spherical fits over one bound data set, each a training (from a
seeded pick or from given rows) and an inner-product assignment of every row,
bit-equal to the oracle's training and assignment, with the rows uploaded once
(the reference's SharedAssigner shares one binding across the fits).
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits

pytestmark = pytest.mark.gpu


def nested_rows(n, d, top, sub, seed):
    """C5's construction, scaled down: top-level means N(0, I), sub-means
    parent + N(0, 0.3^2 I), rows sub-mean + N(0, 0.2^2 I), unit rows."""
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((top, d))
    subs = means[:, None, :] + 0.3 * rng.standard_normal((top, sub, d))
    subs = subs.reshape(top * sub, d)
    x = subs[rng.integers(0, top * sub, n)] + 0.2 * rng.standard_normal((n, d))
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def test_sweep_fits_on_one_binding_equal_the_oracle(engine):
    n, d = 24_000, 96
    x = nested_rows(n, d, 16, 8, 5)
    xb = engine.bind_data(x, d)
    h2d0 = engine.stats()["h2d_bytes"]
    cfg_seed, salt, nepochs = 7, 1, 2.0
    fits = [(16, 0, None), (16, 1, None), (64, 0, None), (64, 1, None),
            (32, 0, np.arange(n)[::97][:32].astype(np.uint32))]
    for k, restart, init_rows in fits:
        seed = eb.seed_for(cfg_seed, salt, k, restart)
        before = engine.stats()["h2d_bytes"]
        tr, labels, scores = engine.fit(xb, d, k, nepochs, seed, init_rows)
        # Only the centroids travel for the assignment: the rows stay bound.
        assert engine.stats()["h2d_bytes"] - before == k * d * 4
        init = None if init_rows is None else x[init_rows[:k]]
        want = oracle.train(x, d, k, nepochs=nepochs, seed=seed, spherical=True, init=init)
        assert np.array_equal(bits(tr.centroids.ravel()), bits(want["centroids"])), (k, restart)
        assert tr.obj == want["obj"]
        wl, ws = oracle.top1(x.ravel(), d, want["centroids"], oracle.IP)
        assert np.array_equal(labels, wl), (k, restart)
        assert np.array_equal(bits(scores), bits(ws)), (k, restart)
    assert engine.stats()["h2d_bytes"] - h2d0 == sum(k * d * 4 for k, _, _ in fits)
    engine.unbind_data()


def test_fit_argument_errors(engine):
    x = nested_rows(1000, 16, 4, 4, 1)
    with pytest.raises(ValueError):
        engine.fit(x, 16, 8, 1.0, 3, np.arange(4))


def test_sweep_picks_and_scores_like_the_oracle(engine):
    """auto::sweep: per k the best of two restarts by mean objective, scored by
    internal_scores; the oracle runs the same sweep on the host."""
    from oracle import metrics as ometrics
    from tests.test_metrics import close

    n, d = 12_000, 64
    x = nested_rows(n, d, 12, 6, 9)
    xb = engine.bind_data(x, d)
    ks, nepochs, seed, salt = (8, 24), 2.0, 11, 2
    picks = [np.random.default_rng(r).permutation(n)[:max(ks)].astype(np.uint32) for r in range(2)]
    got = engine.sweep(xb, d, ks, nepochs, seed, salt, restarts=2, init_rows=picks)
    for (k, scores, tr, labels, sco, obj) in got:
        best = None
        for r in range(2):
            s = eb.seed_for(seed, salt, k, r)
            want = oracle.train(x, d, k, nepochs=nepochs, seed=s, spherical=True,
                                init=x[picks[r][:k]])
            wl, ws = oracle.top1(x.ravel(), d, want["centroids"], oracle.IP)
            o = eb.mean_objective(ws, spherical=True)
            if best is None or o < best[0]:
                best = (o, want, wl, ws)
        o, want, wl, ws = best
        assert obj == o
        assert np.array_equal(bits(tr.centroids.ravel()), bits(want["centroids"]))
        assert np.array_equal(labels, wl) and np.array_equal(bits(sco), bits(ws))
        w = ometrics.internal_scores(x, d, wl, k)
        assert scores["k_eff"] == w["k_eff"]
        assert np.array_equal(scores["sizes"].astype(np.int64), w["sizes"])
        keys = ["silhouette", "calinski_harabasz", "objective"]
        # A one-row cluster's distance to its mean is a cancellation whose value
        # depends on the product's addition order (as in the metrics tests).
        if not np.any(w["sizes"] == 1):
            keys.append("davies_bouldin")
        for key in keys:
            assert close(scores[key], w[key], 1e-6, 1e-9), (k, key, scores[key], w[key])
    engine.unbind_data()
