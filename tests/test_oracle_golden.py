"""Pin the CPU oracle before trusting it.

Golden vectors come from the reference's own Python implementation, run here
by tests/golden/make_golden.py, and (when the reference checkout is present)
from the reference's committed fixture file
crates/emeans-core/tests/fixtures/reference.json, written by the reference's
bench/py/fixtures.py. Tolerances follow the reference's own test
(crates/emeans-core/tests/reference.rs:137-205): split counts and last-pass
labels exact, objective 1e-5 relative, centroids and scores 1e-4.
"""

import json
import math
import os
import pathlib

import numpy as np
import pytest

import oracle

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
# The reference checkout, when the environment names one (EMEANS_REFERENCE):
# its own fixture pins the oracle further; without it those tests skip.
_REF = os.environ.get("EMEANS_REFERENCE")
REF_FIX = pathlib.Path(_REF) / "crates/emeans-core/tests/fixtures" if _REF else None


@pytest.fixture(scope="module")
def golden():
    return json.loads((GOLDEN / "golden.json").read_text())


def ref_fixture():
    if REF_FIX is None:
        pytest.skip("EMEANS_REFERENCE (a reference checkout) is not set")
    p = REF_FIX / "reference.json"
    if not p.exists():
        pytest.skip("reference checkout not present")
    return json.loads(p.read_text())


def check_recipe(c):
    if c.get("law") == "given" or c.get("batch_law") == "given":
        r = oracle.recipe(c["n"], c["k"], c.get("d", 64), 5, "throughput",
                          batch_size=c["given_batch_size"], alpha0=c["given_alpha0"])
    else:
        law = c.get("law", c.get("batch_law"))
        r = oracle.recipe(c["n"], c["k"], c["d"], c["nepochs"], law)
        assert r["epoch_rows"] == c["epoch_rows"], c
        assert r["epoch_steps"] == c["epoch_steps"], c
        assert oracle.unused_threshold(None, c["d"]) == c["unused_threshold"]
    assert r["batch_size"] == c["batch_size"], c
    assert r["alpha0"] == c["alpha0"], c  # bit-exact f64


def test_recipes_bit_exact(golden):
    for c in golden["recipes"]:
        check_recipe(c)


def test_recipes_reference_fixture():
    recs = ref_fixture()["recipes"]
    assert len(recs) > 1400
    for c in recs:
        check_recipe(c)


def test_cosine_schedule_bit_exact(golden):
    for src in (golden["alphas"],):
        for c in src:
            assert oracle.scheduled_alpha(c["alpha0"], c["step"], c["total"]) == c["alpha"]
    for c in ref_fixture()["alphas"]:
        assert oracle.scheduled_alpha(c["alpha0"], c["step"], c["total"]) == c["alpha"]


def check_mt(c):
    if "random_sample" in c:
        got = oracle.random_sample(c["seed"], len(c["random_sample"]))
        assert got.tolist() == c["random_sample"]
        return
    perm = oracle.permutation(c["seed"], c["n"]).astype(np.int64)
    assert perm[:len(c["head"])].tolist() == c["head"]
    if "tail" in c:
        assert perm[len(perm) - len(c["tail"]):].tolist() == c["tail"]
    m = min(c["n"], 5000)
    assert int(perm[:m] @ np.arange(m)) == c["sum"]


def test_mt19937_streams(golden):
    for c in golden["mt19937"]:
        check_mt(c)


def test_mt19937_reference_fixture():
    for c in ref_fixture()["mt19937"]:
        check_mt(c)


def test_fma_chain_known_answers(golden):
    """The top-1 dot is one sequential FMA chain (assign/fused.rs:382-404)."""
    for c in golden["fma_chains"]:
        x = np.array(c["x"], np.float32)
        cc = np.array(c["c"], np.float32)
        d = x.size
        _, s = oracle.top1(x, d, cc, oracle.IP)
        assert s[0] == np.float32(c["dot"]), (d, s[0], c["dot"])


def check_run(c, x):
    d, k = c["d"], c["k"]
    r = oracle.train(x, d, k, nepochs=c["nepochs"], batch_law=c["batch_law"], seed=c["seed"],
                     spherical=c["spherical"])
    assert r["batch_size"] == c["batch_size"]
    assert r["alpha0"] == c["alpha0"]
    assert r["nsplit"] == c["nsplit"], (r["nsplit"], c["nsplit"])
    for got, want in zip(r["obj"], c["obj"]):
        assert abs(got - want) <= 1e-5 * abs(want), (got, want)
    for got, want in zip(r["imbalance"], c["imbalance"]):
        assert abs(got - want) < 1e-9
    assert r["labels"].tolist() == c["labels"]
    want_c = np.array(c["centroids"], np.float32)
    assert np.all(np.abs(r["centroids"] - want_c) <= 1e-4 * np.maximum(np.abs(want_c), 1.0))
    metric = oracle.IP if c["spherical"] else oracle.L2
    lab, sco = oracle.top1(x, d, r["centroids"], metric)
    assert lab.tolist() == c["assign_labels"]
    # Squared distances, or similarities when spherical (e_means.py:638-659).
    want_s = np.array(c["assign_scores"], np.float32)
    assert np.all(np.abs(sco - want_s) <= 1e-4 * np.maximum(np.abs(want_s), 1.0)), \
        np.max(np.abs(sco - want_s))


def test_training_runs_match_reference_python(golden):
    for c in golden["runs"]:
        x = np.fromfile(GOLDEN / f"{c['data']}.f32", dtype="<f4").reshape(c["n"], c["d"])
        check_run(c, x)


def test_training_runs_reference_fixture():
    fx = ref_fixture()
    for c in fx["runs"]:
        x = np.fromfile(REF_FIX / f"{c['data']}.f32", dtype="<f4").reshape(c["n"], c["d"])
        check_run(c, x)


def test_top1_ties_keep_lowest_id():
    """assign/fused.rs:406-420."""
    d = 8
    x = np.ones((3, d), np.float32)
    c = np.zeros((40, d), np.float32)
    for j in (5, 17, 33):
        c[j] = 1.0
    for metric in (oracle.IP, oracle.L2):
        lab, _ = oracle.top1(x, d, c, metric)
        assert lab.tolist() == [5, 5, 5]


def test_top1_against_f64_brute_force():
    """Labels equal f64 brute force except near-ties (core/contract.rs:244-260)."""
    rng = np.random.default_rng(3)
    for n, d, k in [(97, 13, 37), (200, 768, 70), (31, 5, 1), (64, 64, 16)]:
        x = rng.standard_normal((n, d)).astype(np.float32)
        c = rng.standard_normal((k, d)).astype(np.float32)
        for metric in (oracle.IP, oracle.L2):
            lab, sco = oracle.top1(x, d, c, metric)
            x64, c64 = x.astype(np.float64), c.astype(np.float64)
            dots = x64 @ c64.T
            s = dots if metric == oracle.IP else (x64 ** 2).sum(1)[:, None] + \
                (c64 ** 2).sum(1)[None, :] - 2 * dots
            want = s.argmax(1) if metric == oracle.IP else s.argmin(1)
            for i in range(n):
                mag = math.sqrt((x64[i] ** 2).sum() * (c64[want[i]] ** 2).sum()) if \
                    metric == oracle.IP else (x64[i] ** 2).sum() + (c64[want[i]] ** 2).sum()
                mag = max(mag, 1.0)
                if lab[i] != want[i]:
                    assert abs(s[i, lab[i]] - s[i, want[i]]) <= 1e-5 * mag
                assert abs(sco[i] - s[i, lab[i]]) <= 1e-5 * mag


def test_topk_against_f64_with_tie_rule():
    """Best first (score desc, id asc), exclude_self, padding (knn.rs:53-107)."""
    rng = np.random.default_rng(4)
    for m, n, d, kk, ex in [(40, 40, 24, 5, True), (30, 90, 20, 16, False), (9, 7, 33, 10, False)]:
        data = rng.standard_normal((n, d)).astype(np.float32)
        q = data[:m].copy() if ex else rng.standard_normal((m, d)).astype(np.float32)
        ids, sims = oracle.topk(q, data, d, kk, exclude_self=ex)
        ids, sims = ids.reshape(m, kk), sims.reshape(m, kk)
        s64 = q.astype(np.float64) @ data.astype(np.float64).T
        for i in range(m):
            cand = [j for j in range(n) if not (ex and j == i)]
            order = sorted(cand, key=lambda j: (-s64[i, j], j))
            for t in range(kk):
                if t >= len(order):
                    assert ids[i, t] == np.uint32(0xFFFFFFFF) and sims[i, t] == -np.inf
                    continue
                if ids[i, t] != order[t]:
                    assert abs(s64[i, ids[i, t]] - s64[i, order[t]]) <= 1e-5 * max(
                        1.0, float(np.sqrt((q[i].astype(np.float64) ** 2).sum()) ** 2))
            valid = sims[i][ids[i] != 0xFFFFFFFF]
            assert np.all(valid[:-1] >= valid[1:])


def test_scatter_and_ema_float_order():
    """Row-order sums (core/contract.rs:355-392) and the EMA cases (:395-429)."""
    rng = np.random.default_rng(9)
    n, d, k = 500, 20, 37
    x = rng.standard_normal((n, d)).astype(np.float32)
    live = k - k // 5
    labels = ((np.arange(n, dtype=np.uint64) * 2654435761 % 2**32) >> 7) % live
    labels = labels.astype(np.uint32)
    perm = ((np.arange(n) * 31 + 5) % n).astype(np.uint32)
    lo, hi = n // 5, n
    acc0 = ((np.arange(k * d) % 13) * 0.25).astype(np.float32)
    acc = acc0.copy()
    sums, counts = oracle.scatter_add(x.ravel(), d, labels, k, ids=perm, r0=lo, r1=hi, acc=acc)
    want_s = np.zeros((k, d), np.float32)
    want_c = np.zeros(k, np.uint32)
    for p in range(lo, hi):
        want_s[labels[p]] += x[perm[p]]
        want_c[labels[p]] += 1
    assert np.array_equal(counts, want_c)
    assert np.array_equal(sums.view(np.uint32), want_s.ravel().view(np.uint32))
    assert np.array_equal(acc.view(np.uint32), (acc0 + want_s.ravel()).view(np.uint32))
    pos0 = x[:k].ravel().copy()
    for alpha, u0 in [(0.37, 0.8), (1.0, 0.5), (0.9, 0.0)]:
        usage0 = (np.float32(u0) + (np.arange(k) % 5).astype(np.float32) * np.float32(0.125))
        p, u = oracle.ema_update(pos0, usage0, sums, counts, k, d, alpha)
        # numpy restatement of core/cpu.rs:389-432 in float32
        a32, dec = np.float32(alpha), np.float32(1.0 - alpha)
        wu = usage0.copy() if alpha == 1.0 else (usage0 * dec).astype(np.float32)
        wp = pos0.reshape(k, d).copy()
        for j in range(k):
            if counts[j] == 0:
                continue
            cnt = np.float32(counts[j])
            ret = np.float32(0) if alpha == 1.0 else wu[j]
            step = np.float32(a32 * cnt)
            mass = np.float32(ret + step)
            w = np.float32(step / mass)
            mean = (sums.reshape(k, d)[j] / cnt).astype(np.float32)
            wp[j] = mean if w == np.float32(1) else (wp[j] + w * (mean - wp[j])).astype(np.float32)
            wu[j] = mass
        assert np.array_equal(p.view(np.uint32), wp.ravel().view(np.uint32))
        assert np.array_equal(u.view(np.uint32), wu.view(np.uint32))


def test_split_nudges_collapsed_child():
    """apply_splits (core/mod.rs:374-399), including the zero-donor nudge."""
    k, d = 8, 6
    pos = np.arange(k * d, dtype=np.float32) * np.float32(0.37)
    pos[d:2 * d] = 0.0
    usage = (1.0 + np.arange(k) * 0.37).astype(np.float32)
    plan = [(0, 7), (1, 6), (3, 4)]
    p, u = oracle.split(pos, usage, d, plan)
    p = p.reshape(k, d)
    assert p[6, 0] == np.nextafter(np.float32(0), np.float32(1))
    assert u[1] == u[6] == usage[1] / np.float32(2)
    off = np.float32(1e-4) * np.where(np.arange(d) % 2 == 0, 1, -1).astype(np.float32)
    assert np.array_equal(p[0], pos[:d] * (np.float32(1) - off))
    assert np.array_equal(p[7], pos[:d] * (np.float32(1) + off))


def test_normalize_and_norms_float_order():
    rng = np.random.default_rng(2)
    m = rng.standard_normal((50, 37)).astype(np.float32)
    m[0] = 0.0
    m[1] *= np.float32(1e30)
    got = oracle.row_norms(m.ravel(), 37)
    want = np.zeros(50, np.float32)
    for i in range(50):
        s = np.float32(0)
        for v in m[i]:
            s = np.float32(s + np.float32(v * v))
        want[i] = s
    assert np.array_equal(got, want)
    u = oracle.normalize_rows(m.ravel(), 37).reshape(50, 37)
    assert np.all(u[0] == 0)
    n64 = np.linalg.norm(m[2:].astype(np.float64), axis=1)
    assert np.allclose(u[2:], m[2:] / n64[:, None], rtol=1e-5, atol=1e-6)


def test_self_join_rows_equal_the_full_self_join():
    """oracle.topk_self_rows (the self-join for a block of query rows, the
    bench's subsample check) equals those rows of the full self-join."""
    rng = np.random.default_rng(4)
    n, d, kk = 700, 24, 7
    x = rng.standard_normal((n, d)).astype(np.float32)
    x[600:610] = x[5:15]  # duplicates: equal scores keep the lower id
    ids, sims = oracle.topk(x, x, d, kk, exclude_self=True)
    for q0, m in ((0, 50), (333, 120), (650, 50)):
        si, ss = oracle.topk_self_rows(x, d, q0, m, kk)
        assert np.array_equal(si, ids[q0 * kk:(q0 + m) * kk])
        assert np.array_equal(ss.view(np.uint32), sims[q0 * kk:(q0 + m) * kk].view(np.uint32))
