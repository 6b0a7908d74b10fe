"""The device loop on the B200 against the oracle's device loop, bit for bit,
and against the reference Python runs (the golden vectors).

Both run the reference's float order for every op (core/train.rs:60-303), so
the labels, centroids, masses and per-epoch objectives must be identical.
Against the faiss NumpyEmeans runs the reference's own tolerances apply
(crates/emeans-core/tests/reference.rs:137-205).
"""

import json
import pathlib

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, mixture

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def same_run(got: eb.Trained, want: dict):
    assert got.batch_size == want["batch_size"] and got.alpha0 == want["alpha0"]
    assert got.nsplit == want["nsplit"]
    assert got.obj == want["obj"], (got.obj, want["obj"])
    assert got.imbalance == want["imbalance"]
    assert np.array_equal(got.labels, want["labels"])
    assert np.array_equal(bits(got.centroids.ravel()), bits(want["centroids"]))
    assert np.array_equal(bits(got.positions.ravel()), bits(want["positions"]))
    assert np.array_equal(bits(got.usage), bits(want["usage"]))


def test_golden_runs(engine):
    g = json.loads((GOLDEN / "golden.json").read_text())
    for c in g["runs"]:
        x = np.fromfile(GOLDEN / f"{c['data']}.f32", dtype="<f4").reshape(c["n"], c["d"])
        cfg = eb.Config(d=c["d"], k=c["k"], nepochs=c["nepochs"], batch_law=c["batch_law"],
                        seed=c["seed"], spherical=c["spherical"])
        got = engine.train(x, cfg)
        want = oracle.train(x, c["d"], c["k"], nepochs=c["nepochs"], batch_law=c["batch_law"],
                            seed=c["seed"], spherical=c["spherical"])
        same_run(got, want)
        # The reference Python run (reference.rs:160-204 tolerances).
        assert got.nsplit == c["nsplit"]
        assert got.labels.tolist() == c["labels"]
        for a, b in zip(got.obj, c["obj"]):
            assert abs(a - b) <= 1e-5 * abs(b)
        wc = np.array(c["centroids"], np.float32)
        assert np.all(np.abs(got.centroids.ravel() - wc) <= 1e-4 * np.maximum(np.abs(wc), 1))
        metric = eb.IP if c["spherical"] else eb.L2
        lab, sco = engine.assign(x, c["d"], got.centroids, metric)
        assert lab.tolist() == c["assign_labels"]


def test_config1_spherical_cpu_config(engine):
    """spherical, n=20,000, d=64, k=32, seed 7."""
    rng = np.random.default_rng(7)
    means = rng.standard_normal((32, 64))
    means /= np.linalg.norm(means, axis=1, keepdims=True)
    x = means[rng.integers(0, 32, 20000)] + 0.3 * rng.standard_normal((20000, 64))
    x = (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)
    cfg = eb.Config(d=64, k=32, spherical=True, seed=7)
    got = engine.train(x, cfg)
    want = oracle.train(x, 64, 32, spherical=True, seed=7)
    assert got.batch_size == 1024 and got.total_steps == 100
    same_run(got, want)


def test_l2_with_revival_and_fractional_epochs(engine):
    x = mixture(6000, 48, 30, 0.4, False, 21)
    cfg = eb.Config(d=48, k=96, nepochs=2.5, seed=5)
    got = engine.train(x, cfg)
    want = oracle.train(x, 48, 96, nepochs=2.5, seed=5)
    same_run(got, want)
    assert got.n_splits > 0


def test_resume_from_state(engine):
    x = mixture(4000, 24, 12, 0.5, False, 8)
    first = engine.train(x, eb.Config(d=24, k=16, nepochs=1, seed=3))
    got = engine.train(x, eb.Config(d=24, k=16, nepochs=2, seed=4),
                       state=(first.positions, first.usage))
    want = oracle.train(x, 24, 16, nepochs=2, seed=4,
                        state=(first.positions.ravel(), first.usage))
    same_run(got, want)


def test_train_argument_errors(engine):
    x = np.ones((10, 4), np.float32)
    with pytest.raises(eb.EngineError, match="at least k"):
        engine.train(x, eb.Config(d=4, k=11))
    with pytest.raises(eb.EngineError, match="finite"):
        engine.train(x, eb.Config(d=4, k=2), init=np.full((2, 4), np.nan, np.float32))


def test_training_on_bound_rows(engine):
    """Rows bound with Assigner::bind_data are trained on in place (no upload
    inside the run); the result is the same as a run that uploads them."""
    x = mixture(12000, 96, 30, 0.4, False, 21)
    cfg = eb.Config(d=96, k=120, seed=4, spherical=False, nepochs=3.0)
    want = engine.train(x, cfg)
    engine.bind_data(x, 96)
    try:
        got = engine.train(x, cfg)
        again = engine.train(x, cfg)
    finally:
        engine.unbind_data()
    for g in (got, again):
        assert np.array_equal(bits(g.centroids.ravel()), bits(want.centroids.ravel()))
        assert np.array_equal(g.labels, want.labels) and g.obj == want.obj


def test_config2_training_and_final_assign(engine):
    """BASELINE config 2, the headline run at full size: 200,000 x 768 L2,
    k = 1024, seed 0, the reference schedule (65 steps of 16,384 rows), then
    the full-data final assign. Labels, centroids, masses and every epoch's
    objective are bit-equal to the oracle's training, and the final assign's
    labels and scores to the oracle's top-1."""
    from bench import gen_rows

    n, d, k = 200_000, 768, 1024
    x = gen_rows(n, d, 0)
    cfg = eb.Config(d=d, k=k, seed=0, spherical=False)
    engine.bind_data(x, d)
    try:
        got = engine.train(x, cfg)
        lab, sco = engine.assign(x, d, got.centroids, eb.L2)
    finally:
        engine.unbind_data()
    want = oracle.train(x, d, k, seed=0)
    assert got.total_steps == 65 and got.batch_size == 16384
    same_run(got, want)
    wl, ws = oracle.top1(x.ravel(), d, want["centroids"], oracle.L2)
    assert np.array_equal(lab, wl)
    assert np.array_equal(bits(sco), bits(ws))
