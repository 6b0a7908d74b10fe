"""Internal clustering scores (metrics::internal_scores, crates/emeans-cluster/
src/metrics.rs:115-274): the oracle pinned to scikit-learn fixtures on the
CPU (the reference test's tolerance, relative 1e-5), and the device path
(eb_internal_scores) against the oracle on a GPU.

The n x k_eff product is FP32 on both sides in different addition orders (FMA
chains on the device's SIMT path, split FP16 products with FP32 accumulation
on its tensor-core path, the BLAS order in the oracle, the gemm crate's in the
reference), so the scores agree to rounding: relative 1e-6 here, on both
device paths (screen mode 0: SIMT; 2: tensor cores). Counts and k_eff are
exact."""
import json
import os

import numpy as np
import pytest

import emeans_b200 as eb
from oracle.metrics import internal_scores as oracle_scores

HERE = os.path.dirname(os.path.abspath(__file__))
KEYS = ("silhouette", "calinski_harabasz", "davies_bouldin")


def fixtures():
    with open(os.path.join(HERE, "golden", "metrics.json")) as f:
        for c in json.load(f)["cases"]:
            x = np.fromfile(os.path.join(HERE, "golden", f"metrics_{c['name']}.f32"), "<f4")
            yield c, x


def close(a, b, rel, abs_=1e-12):
    return abs(a - b) <= rel * max(abs(b), abs_)


def test_oracle_matches_scikit_learn():
    n_cases = 0
    for c, x in fixtures():
        r = oracle_scores(x, c["d"], c["labels"], c["k"])
        for key in KEYS:
            assert close(r[key], c[key], 1e-5), (c["name"], key, r[key], c[key])
        assert r["k_eff"] == len(set(c["labels"]))
        n_cases += 1
    assert n_cases == 3


def test_oracle_degenerate_cases():
    x = np.eye(4, dtype=np.float32)
    r = oracle_scores(x, 4, [2, 2, 2, 2], 3)
    assert r["k_eff"] == 1 and r["silhouette"] == 0.0
    assert r["calinski_harabasz"] == 0.0 and r["davies_bouldin"] == 0.0
    r = oracle_scores(np.zeros(0, np.float32), 4, [], 3)
    assert r["k_eff"] == 0 and r["objective"] == 0.0


def test_null_engine_is_invalid():
    lib = eb.load()
    assert lib.eb_internal_scores(None, None, 0, 4, None, 1, None, None) == eb.INVALID_ARGUMENT


def unit_rows(rng, n, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def nearest_labels(x, c):
    return np.argmax(x @ c.T, axis=1).astype(np.uint32)


def check(got, want, rel=1e-6):
    assert got["k_eff"] == want["k_eff"]
    assert np.array_equal(got["sizes"].astype(np.int64), want["sizes"])
    for key in KEYS + ("objective",):
        assert close(got[key], want[key], rel, 1e-9), (key, got[key], want[key])


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 2], ids=["simt", "tensor"])
def test_device_matches_oracle_and_scikit_learn_on_fixtures(mode):
    with eb.Engine(0) as e:
        e.set_screen_mode(mode)
        for c, x in fixtures():
            got = e.internal_scores(x, c["d"], c["labels"], c["k"])
            check(got, oracle_scores(x, c["d"], c["labels"], c["k"]))
            for key in KEYS:
                assert close(got[key], c[key], 1e-5), (c["name"], key)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 2], ids=["simt", "tensor"])
@pytest.mark.parametrize("n,d,k", [(1000, 64, 17), (777, 33, 50), (4096, 96, 130), (130, 8, 3),
                                   (3000, 48, 700)])
def test_device_matches_oracle(n, d, k, mode):
    rng = np.random.default_rng(n + d + k)
    x = unit_rows(rng, n, d)
    c = unit_rows(rng, k, d)
    lab = nearest_labels(x, c)
    lab[lab == 1] = 0          # label 1 empty
    lab[lab == k - 2] = 0      # label k - 2: two rows
    lab[10:12] = k - 2
    lab[:3] = k - 1            # a small cluster at the last label
    # (No singleton here: a one-row cluster's distance to its mean is the
    # square root of a cancellation of FP32 products, whose value depends on
    # the product's addition order; Davies-Bouldin would compare those.)
    with eb.Engine(0) as e:
        e.set_screen_mode(mode)
        check(e.internal_scores(x, d, lab, k), oracle_scores(x, d, lab, k))


@pytest.mark.gpu
def test_device_degenerate_cases():
    rng = np.random.default_rng(5)
    x = unit_rows(rng, 300, 16)
    with eb.Engine(0) as e:
        one = e.internal_scores(x, 16, np.full(300, 4, np.uint32), 9)
        assert one["k_eff"] == 1 and one["silhouette"] == 0.0
        assert one["calinski_harabasz"] == 0.0 and one["davies_bouldin"] == 0.0
        check(one, oracle_scores(x, 16, np.full(300, 4), 9))
        empty = e.internal_scores(np.zeros(0, np.float32), 16, np.zeros(0, np.uint32), 9)
        assert empty["k_eff"] == 0 and empty["silhouette"] == 0.0 and empty["objective"] == 0.0
        with pytest.raises(eb.EngineError, match="label out of range"):
            e.internal_scores(x, 16, np.full(300, 9, np.uint32), 9)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["simt", "auto", "tensor"])
def test_device_bound_rows_and_larger_case(mode):
    """Rows given, then bound (read in place; after an assign on them, the
    tensor-core path reads their split copy too)."""
    rng = np.random.default_rng(8)
    n, d, k = 20000, 256, 300
    x = unit_rows(rng, n, d)
    c = unit_rows(rng, k, d)
    lab = nearest_labels(x, c)
    want = oracle_scores(x, d, lab, k)
    with eb.Engine(0) as e:
        e.set_screen_mode(mode)
        check(e.internal_scores(x, d, lab, k), want)
        e.bind_data(x, d)
        check(e.internal_scores(x, d, lab, k), want)
        e.assign(x, d, c, eb.IP, ids=np.arange(n, dtype=np.uint32))
        check(e.internal_scores(x, d, lab, k), want)
