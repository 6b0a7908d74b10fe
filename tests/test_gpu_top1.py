"""Top-1 on the B200 against the CPU oracle: labels and scores bit-equal.

The oracle follows the reference CPU kernel's float order (one sequential FMA
chain per dot, crates/emeans-core/src/assign/fused.rs:12-16), so the engine
must reproduce every bit, whether a row was certified by the tensor-core
screen or scanned exactly. Shapes follow the reference contract suite
(crates/emeans-core/src/core/contract.rs:75-161): check() shapes with
indexed and dense selections and a sub-range whose outside must stay
untouched, check_production() (16,384 x 768, k 1024 / 1000 with duplicate
centroids in other tiles), and adversarial near-ties.
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, contract_centroids, mixture, near_tie_centroids, \
    production_centroids

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[0, 2], ids=["exact", "screen"])
def eng(engine, request):
    """The session engine on the exact SIMT path (0) or the tcgen05 screen (2)."""
    engine.set_screen_mode(request.param)
    yield engine
    engine.set_screen_mode(1)

SHAPES = [(1000, 768, 64), (777, 768, 100), (513, 13, 70), (2000, 20, 300), (300, 64, 1),
          (600, 768, 1024)]


def run_top1(engine, x, c, metric, ids=None, lo=None, hi=None):
    n, d = x.shape
    k = c.shape[0]
    m = n if ids is None else len(ids)
    lo = 0 if lo is None else lo
    hi = m if hi is None else hi
    xb = engine.bind(x, d)
    cb = engine.upload_f32(c)
    cn = None
    if metric == eb.L2:
        cn = engine.zeros_f32(k)
        engine.row_norms(cb, k, d, cn)
    ib = engine.upload_u32(ids) if ids is not None else None
    lab = engine.upload_u32(np.full(m, 0xFFFFFFFF, np.uint32))
    sco = engine.upload_f32(np.full(m, np.nan, np.float32))
    engine.top1(xb, d, ib, range(lo, hi), cb, cn, k, metric, lab, sco)
    return lab.read(), sco.read()


def check_against_oracle(engine, x, c, metric, ids=None, lo=None, hi=None):
    n, d = x.shape
    m = n if ids is None else len(ids)
    lo = 0 if lo is None else lo
    hi = m if hi is None else hi
    gl, gs = run_top1(engine, x, c, metric, ids, lo, hi)
    wl = np.full(m, 0xFFFFFFFF, np.uint32)
    ws = np.full(m, np.nan, np.float32)
    oracle.top1(x.ravel(), d, c.ravel(), metric, ids=ids, r0=lo, r1=hi, labels=wl, scores=ws)
    outside = np.ones(m, bool)
    outside[lo:hi] = False
    assert np.all(gl[outside] == 0xFFFFFFFF) and np.all(np.isnan(gs[outside])), \
        "top1 wrote outside the selection"
    bad = np.flatnonzero(gl[lo:hi] != wl[lo:hi])
    assert bad.size == 0, f"{bad.size} labels differ, first at {lo + bad[0]}"
    assert np.array_equal(bits(gs[lo:hi]), bits(ws[lo:hi]))


@pytest.mark.parametrize("n,d,k", SHAPES)
@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_contract_shapes(eng, n, d, k, metric):
    x = mixture(n, d, 11, 0.6, metric == eb.IP, 3 * n + k)
    c = contract_centroids(x, d, k)
    perm = ((np.arange(n, dtype=np.int64) * 7919 + 13) % n).astype(np.uint32)
    lo, hi = n // 7, n - n // 9
    check_against_oracle(eng, x, c, metric, ids=perm, lo=lo, hi=hi)
    check_against_oracle(eng, x, c, metric, lo=lo, hi=hi)


@pytest.mark.parametrize("k", [1024, 1000])
@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_production_batch_with_duplicate_centroids(eng, k, metric):
    n, d = 16384, 768
    x = mixture(n, d, 64, 0.6, metric == eb.IP, 5 * n + k)
    c = production_centroids(x, k)
    check_against_oracle(eng, x, c, metric)
    # Exact duplicates: the lower id wins.
    gl, _ = run_top1(eng, x, c, metric)
    assert np.all(gl < k - 256)


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_screen_runs_on_large_calls(engine, metric):
    """Auto mode takes the tensor-core path for a production batch; few rows fall back."""
    engine.set_screen_mode(1)
    n, d, k = 16384, 768, 1024
    x = mixture(n, d, 64, 0.6, metric == eb.IP, 99)
    c = production_centroids(x, k)
    s0 = engine.stats()
    check_against_oracle(engine, x, c, metric)
    s1 = engine.stats()
    screened = s1["screened_rows"] - s0["screened_rows"]
    fallback = s1["fallback_rows"] - s0["fallback_rows"]
    print(f"screened {screened} rows, {fallback} fell back, "
          f"{s1['rescored_candidates'] - s0['rescored_candidates']} candidates re-scored")
    assert screened == n
    assert fallback < n // 2


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_near_ties_and_scaled_rows(eng, metric):
    n, d, k = 4096, 256, 512
    c = near_tie_centroids(d, k, 3)
    rng = np.random.default_rng(8)
    x = (c[rng.integers(0, k, n)] + np.float32(1e-3) * rng.standard_normal((n, d))).astype(np.float32)
    scale = np.array([1.0, 1e3, 1e-3, 1e-15], np.float32)[np.arange(n) % 4]
    x = (x * scale[:, None]).astype(np.float32)
    check_against_oracle(eng, x, c, metric)


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_odd_shapes(eng, metric):
    rng = np.random.default_rng(0)
    for n, d, k in [(1, 1, 1), (5, 3, 2), (129, 17, 257), (64, 8, 40), (200, 100, 3)]:
        x = rng.standard_normal((n, d)).astype(np.float32)
        c = rng.standard_normal((k, d)).astype(np.float32)
        check_against_oracle(eng, x, c, metric)


def test_ties_keep_the_lowest_id(eng):
    d = 8
    x = np.ones((3, d), np.float32)
    c = np.zeros((40, d), np.float32)
    for j in (5, 17, 33):
        c[j] = 1.0
    for metric in (eb.IP, eb.L2):
        gl, _ = run_top1(eng, x, c, metric)
        assert gl.tolist() == [5, 5, 5]


def test_nonfinite_rows_follow_the_cpu_semantics(eng):
    d, k = 16, 9
    rng = np.random.default_rng(1)
    x = rng.standard_normal((6, d)).astype(np.float32)
    x[1, 3] = np.nan
    x[2, 0] = np.inf
    x[3] = 0.0
    c = rng.standard_normal((k, d)).astype(np.float32)
    c[4, 2] = np.nan
    for metric in (eb.IP, eb.L2):
        check_against_oracle(eng, x, c, metric)


def test_bad_row_id_is_an_error(eng):
    d = 4
    x = np.ones((10, d), np.float32)
    c = np.ones((3, d), np.float32)
    xb = eng.bind(x, d)
    cb = eng.upload_f32(c)
    ib = eng.upload_u32(np.array([0, 1, 99], np.uint32))
    lab, sco = eng.zeros_u32(3), eng.zeros_f32(3)
    eng.top1(xb, d, ib, range(0, 3), cb, None, 3, eb.IP, lab, sco)
    with pytest.raises(eb.EngineError) as ei:
        eng.sync()
    assert ei.value.code == eb.INVALID_ARGUMENT
    eng.sync()


def test_argument_checks(eng):
    d = 4
    xb = eng.bind(np.ones((10, d), np.float32), d)
    cb = eng.upload_f32(np.ones((3, d), np.float32))
    lab, sco = eng.zeros_u32(10), eng.zeros_f32(10)
    with pytest.raises(eb.EngineError, match="past the data"):
        eng.top1(xb, d, None, range(0, 11), cb, None, 3, eb.IP, lab, sco)
    with pytest.raises(eb.EngineError, match="centroid norms"):
        eng.top1(xb, d, None, range(0, 10), cb, None, 3, eb.L2, lab, sco)
    with pytest.raises(eb.EngineError, match="k x d"):
        eng.top1(xb, d, None, range(0, 10), cb, None, 4, eb.IP, lab, sco)


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_assign_host_api(eng, metric):
    n, d, k = 3000, 96, 130
    x = mixture(n, d, 20, 0.5, metric == eb.IP, 77)
    c = contract_centroids(x, d, k)
    gl, gs = eng.assign(x, d, c, metric)
    wl, ws = oracle.top1(x.ravel(), d, c.ravel(), metric)
    assert np.array_equal(gl, wl) and np.array_equal(bits(gs), bits(ws))
    ids = np.random.default_rng(2).permutation(n)[:777].astype(np.uint32)
    eng.bind_data(x, d)
    gl, gs = eng.assign(eng._bound, d, c, metric, ids=ids)
    eng.unbind_data()
    wl, ws = oracle.top1(x.ravel(), d, c.ravel(), metric, ids=ids)
    assert np.array_equal(gl, wl) and np.array_equal(bits(gs), bits(ws))


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_assign_pinned_buffers_in_slices(engine, metric):
    """eb_assign with pinned host buffers and enough rows (70,000) for the
    sliced path: three large slices and a small last one, each slice's labels
    and scores copied back as soon as they are ready."""
    import torch

    n, d, k = 70000, 64, 300
    x = mixture(n, d, 40, 0.5, metric == eb.IP, 91)
    c = contract_centroids(x, d, k)
    hx = torch.from_numpy(x).pin_memory()
    hc = torch.from_numpy(np.ascontiguousarray(c)).pin_memory()
    hl = torch.empty(n, dtype=torch.int32).pin_memory()
    hs = torch.empty(n, dtype=torch.float32).pin_memory()
    engine.assign_ptr(hx.data_ptr(), n, d, hc.data_ptr(), k, metric, hl.data_ptr(),
                      hs.data_ptr())
    wl, ws = oracle.top1(x.ravel(), d, c.ravel(), metric)
    assert np.array_equal(hl.numpy().view(np.uint32), wl)
    assert np.array_equal(bits(hs.numpy()), bits(ws))
    gl, gs = engine.assign(x, d, c, metric)  # pageable buffers: results at the end
    assert np.array_equal(gl, wl) and np.array_equal(bits(gs), bits(ws))


@pytest.mark.parametrize("metric", [eb.IP, eb.L2])
def test_assign_only_config_shape(engine, metric):
    """The assign-only config's shape, scaled in rows: unit rows and k = 65,536
    unit centroids drawn the same way, d = 1024 (256 centroid tiles per row
    tile, candidate lists compacted many times)."""
    engine.set_screen_mode(1)
    d, k, n = 1024, 65536, 3000
    rng = np.random.default_rng(1)
    c = rng.standard_normal((k, d), dtype=np.float32)
    c /= np.linalg.norm(c, axis=1, keepdims=True)
    x = rng.standard_normal((n, d), dtype=np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    s0 = engine.stats()
    check_against_oracle(engine, x, c, metric)
    s1 = engine.stats()
    assert s1["screened_rows"] - s0["screened_rows"] == n


def test_a_screen_wait_that_runs_out_is_reported_and_results_stay_exact(engine):
    """Failure detection without a fault: the test hook makes the screen's
    first CTA wait, at its second centroid tile, on a device barrier that
    nothing arrives at. The wait gives up after its limit (2 s); the CTA's
    copies and products in flight land before it frees its tensor memory and
    exits; its rows take the exact full scan. The next synchronising call
    reports the timeout (EB_ERROR), the labels and scores still equal the
    oracle's, and the engine keeps working."""
    n, d, k = 3000, 96, 700  # 24 row tiles, three 256-centroid tiles each
    x = mixture(n, d, 16, 0.5, False, 12)
    c = contract_centroids(x, d, k)
    wl, ws = oracle.top1(x.ravel(), d, c.ravel(), oracle.L2)
    engine.set_screen_mode(2)
    try:
        xb, cb, cn = engine.bind(x, d), engine.upload_f32(c), engine.zeros_f32(k)
        engine.row_norms(cb, k, d, cn)
        lab, sco = engine.zeros_u32(n), engine.zeros_f32(n)
        fb0 = engine.stats()["fallback_rows"]
        assert eb.load().eb_test_screen_dead_wait(engine.h, 1) == eb.OK
        engine.top1(xb, d, None, range(0, n), cb, cn, k, eb.L2, lab, sco)
        with pytest.raises(eb.EngineError, match="wait timed out") as err:
            engine.sync()
        assert err.value.code == eb.ERROR
        assert np.array_equal(lab.read(), wl)
        assert np.array_equal(bits(sco.read()), bits(ws))
        assert engine.stats()["fallback_rows"] - fb0 >= 128  # CTA 0's row tile
        # The hook cleared itself: the same call again is clean and exact.
        lab2, sco2 = engine.zeros_u32(n), engine.zeros_f32(n)
        engine.top1(xb, d, None, range(0, n), cb, cn, k, eb.L2, lab2, sco2)
        engine.sync()
        assert np.array_equal(lab2.read(), wl)
        assert np.array_equal(bits(sco2.read()), bits(ws))
    finally:
        engine.set_screen_mode(1)


@pytest.mark.parametrize("m,k", [(6000, 1024), (600, 1024), (3000, 700), (2000, 1300),
                                 (9000, 1024), (300, 257)])
@pytest.mark.parametrize("metric", [eb.L2, eb.IP])
def test_row_tiles_split_over_centroid_parts(engine, m, k, metric):
    """Calls with few row tiles spread each row tile's centroid tiles over 2
    or 4 parts (each part keeps its own candidate lists, merged by the
    collect step); uneven parts (3 and 6 centroid tiles) included. Labels and
    scores stay bit-equal to the oracle."""
    d = 96
    x = mixture(m, d, 20, 0.4, metric == eb.IP, m + k)
    c = contract_centroids(x, d, k)
    engine.set_screen_mode(2)
    try:
        gl, gs = run_top1(engine, x, c, metric)
    finally:
        engine.set_screen_mode(1)
    wl, ws = oracle.top1(x.ravel(), d, c.ravel(), metric)
    assert np.array_equal(gl, wl)
    assert np.array_equal(bits(gs), bits(ws))
