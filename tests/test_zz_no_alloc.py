"""The allocation-free exact top-1 (eb_top1_exact_noalloc) through the C ABI.

The entry point is for callers that cannot allocate device memory while a
call runs (a server that reserves its memory once at start-up and keeps a
fixed footprint per request, or a caller on a latency budget that cannot take
an allocation's pause). Checked against eb_top1 on the exact SIMT path and
against the CPU oracle (the reference's fused float order): the same labels
and scores bit for bit, on two calls in a row (the second reuses the device's
fixed scratch), for both metrics, dense and indexed selections; a call leaves
the engine's device-allocation count unchanged; sizes the kernel cannot index
are refused before any launch. The file is named to run after the other GPU
tests, so it also covers a process whose engine and library have already done
other work.
"""

import ctypes as C

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, contract_centroids, mixture

pytestmark = pytest.mark.gpu

MAX_ROWS = 1048576  # EB_NOALLOC_MAX_ROWS


def noalloc_fn():
    f = eb.load().eb_top1_exact_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                  C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p,
                  C.c_void_p]
    return f


def call_noalloc(engine, xb, n, d, ib, lo, hi, cb, cn, k, metric, lab, sco):
    rc = noalloc_fn()(engine.h, xb.ptr, n, d, ib.ptr if ib is not None else None, lo, hi,
                      cb.ptr, cn.ptr if cn is not None else None, k, metric, lab.ptr, sco.ptr)
    return rc


@pytest.mark.parametrize("metric", [eb.L2, eb.IP])
def test_matches_top1_on_two_calls_in_a_row(engine, metric):
    engine.set_screen_mode(0)
    try:
        for call, (n, d, k, use_ids) in enumerate([(5000, 96, 300, False),
                                                  (3001, 40, 77, True)]):
            x = mixture(n, d, 12, 0.5, metric == eb.IP, 41 + call)
            c = contract_centroids(x, d, k)
            xb = engine.bind(x, d)
            cb = engine.upload_f32(c)
            cn = None
            if metric == eb.L2:
                cn = engine.zeros_f32(k)
                engine.row_norms(cb, k, d, cn)
            ids = None
            m = n
            if use_ids:
                ids = np.random.default_rng(call).permutation(n)[: n - 500].astype(np.uint32)
                m = ids.size
            ib = engine.upload_u32(ids) if ids is not None else None
            lo, hi = m // 5, m - 3
            want_l = engine.upload_u32(np.full(m, 0xFFFFFFFF, np.uint32))
            want_s = engine.upload_f32(np.full(m, np.nan, np.float32))
            engine.top1(xb, d, ib, range(lo, hi), cb, cn, k, metric, want_l, want_s)
            got_l = engine.upload_u32(np.full(m, 0xFFFFFFFF, np.uint32))
            got_s = engine.upload_f32(np.full(m, np.nan, np.float32))
            rc = call_noalloc(engine, xb, n, d, ib, lo, hi, cb, cn, k, metric, got_l, got_s)
            assert rc == eb.OK, eb.load().eb_last_error().decode()
            engine.sync()
            wl, ws, gl, gs = want_l.read(), want_s.read(), got_l.read(), got_s.read()
            assert np.array_equal(gl, wl), f"call {call}: labels differ"
            assert np.array_equal(bits(gs), bits(ws)), f"call {call}: scores differ"
            assert np.all(gl[:lo] == 0xFFFFFFFF) and np.all(gl[hi:] == 0xFFFFFFFF)
            # The CPU oracle on the same selected rows.
            sel = (ids[lo:hi].astype(np.int64) if ids is not None else np.arange(lo, hi))
            ol, osc = oracle.top1(x[sel].ravel(), d, c.ravel(), metric)
            assert np.array_equal(gl[lo:hi], ol), f"call {call}: labels differ from the oracle"
            assert np.array_equal(bits(gs[lo:hi]), bits(osc)), \
                f"call {call}: scores differ from the oracle"
    finally:
        engine.set_screen_mode(1)


def test_rejects_a_selection_over_the_limit(engine):
    d, k = 4, 3
    xb = engine.bind(np.ones((8, d), np.float32), d)
    cb = engine.upload_f32(np.ones((k, d), np.float32))
    ib = engine.upload_u32(np.zeros(MAX_ROWS + 1, np.uint32))
    lab, sco = engine.zeros_u32(8), engine.zeros_f32(8)
    rc = call_noalloc(engine, xb, 8, d, ib, 0, MAX_ROWS + 1, cb, None, k, eb.IP, lab, sco)
    assert rc == eb.INVALID_ARGUMENT
    assert "at most 1048576 rows" in eb.load().eb_last_error().decode()
    engine.sync()


def test_a_call_allocates_no_device_memory(engine):
    """After the set-up call, an L2 call on a selection larger than any other
    in this file leaves the engine's device-allocation count unchanged."""
    n, d, k = 300_000, 64, 50
    x = mixture(n, d, 9, 0.5, False, 77)
    c = contract_centroids(x, d, k)
    xb = engine.bind(x, d)
    cb = engine.upload_f32(c)
    cn = engine.zeros_f32(k)
    engine.row_norms(cb, k, d, cn)
    lab, sco = engine.zeros_u32(n), engine.zeros_f32(n)
    assert call_noalloc(engine, xb, n, d, None, 0, 64, cb, cn, k, eb.L2, lab, sco) == eb.OK
    engine.sync()
    before = engine.device_allocations()
    rc = call_noalloc(engine, xb, n, d, None, 0, n, cb, cn, k, eb.L2, lab, sco)
    assert rc == eb.OK, eb.load().eb_last_error().decode()
    engine.sync()
    assert engine.device_allocations() == before
    wl, ws = oracle.top1(x[:4096].ravel(), d, c.ravel(), eb.L2)
    assert np.array_equal(lab.read(0, 4096), wl)
    assert np.array_equal(bits(sco.read(0, 4096)), bits(ws))


def test_rejects_sizes_the_kernel_cannot_index(engine):
    """d past 2^31 - 1 and n * d past the long range are refused up front (no
    launch: the pointers are never read)."""
    xb = engine.bind(np.ones((8, 4), np.float32), 4)
    cb = engine.upload_f32(np.ones((3, 4), np.float32))
    lab, sco = engine.zeros_u32(8), engine.zeros_f32(8)
    rc = call_noalloc(engine, xb, 8, 2 ** 31, None, 0, 8, cb, None, 3, eb.IP, lab, sco)
    assert rc == eb.INVALID_ARGUMENT
    assert "d must be at most" in eb.load().eb_last_error().decode()
    rc = call_noalloc(engine, xb, 2 ** 62, 4, None, 0, 8, cb, None, 3, eb.IP, lab, sco)
    assert rc == eb.INVALID_ARGUMENT
    assert "n * d overflows" in eb.load().eb_last_error().decode()
    engine.sync()
