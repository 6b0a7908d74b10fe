"""Parity of the update ops on the B200 against the CPU oracle, bit for bit.

Cases follow the reference contract suite (crates/emeans-core/src/core/contract.rs):
check_scatter_ema (:355-498) and check_norms (:500-553) on the check()
shapes, plus the production batch (16,384 x 768, k = 1024) with Zipf labels.
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, mixture

pytestmark = pytest.mark.gpu

# (20000, 96, 32) and (12000, 768, 40) average hundreds of rows a centroid
# (the staged sum's full-pass shape; the others take its training-batch
# shape). With k <= 1024 the label order ranks 2,048-position blocks
# ((9000, 40, 700): several blocks and a ragged last one); (5000, 24, 1500)
# and (3000, 8, 2048) take the larger-k order (256-position warp segments
# counted in global memory).
SHAPES = [(1000, 768, 64), (777, 768, 100), (513, 13, 70), (2000, 20, 300), (300, 64, 1),
          (600, 768, 1024), (20000, 96, 32), (12000, 768, 40), (9000, 40, 700),
          (5000, 24, 1500), (3000, 8, 2048)]


@pytest.mark.parametrize("n,d,k", SHAPES)
def test_scatter_add_bit_equal(engine, n, d, k):
    k = min(k, n)
    x = mixture(n, d, 7, 0.5, False, n + d)
    live = max(k - k // 5, 1)
    labels = (((np.arange(n, dtype=np.uint64) * 2654435761) % 2**32) >> 7) % live
    labels = labels.astype(np.uint32)
    perm = ((np.arange(n, dtype=np.int64) * 31 + 5) % n).astype(np.uint32)
    lo, hi = n // 5, n
    acc0 = ((np.arange(k * d) % 13) * 0.25).astype(np.float32)
    xb = engine.bind(x, d)
    ids = engine.upload_u32(perm)
    lab = engine.upload_u32(labels)
    sums = engine.upload_f32(np.full(k * d, 7.0, np.float32))
    counts = engine.upload_u32(np.full(k, 3, np.uint32))
    acc = engine.upload_f32(acc0)
    engine.scatter_add(xb, d, ids, range(lo, hi), lab, k, sums, counts, acc)
    acc_w = acc0.copy()
    ws, wc = oracle.scatter_add(x.ravel(), d, labels, k, ids=perm, r0=lo, r1=hi, acc=acc_w)
    assert np.array_equal(counts.read(), wc)
    assert np.array_equal(bits(sums.read()), bits(ws))
    assert np.array_equal(bits(acc.read()), bits(acc_w))


def test_scatter_add_production_batch_dense_and_empty(engine):
    n, d, k = 16384, 768, 1024
    x = mixture(n, d, 64, 0.6, True, 11)
    rng = np.random.default_rng(1)
    w = 1.0 / np.arange(1, k + 1) ** 1.1
    labels = rng.choice(k, n, p=w / w.sum()).astype(np.uint32)
    xb = engine.bind(x, d)
    lab = engine.upload_u32(labels)
    sums, counts = engine.zeros_f32(k * d), engine.zeros_u32(k)
    engine.scatter_add(xb, d, None, range(0, n), lab, k, sums, counts)
    ws, wc = oracle.scatter_add(x.ravel(), d, labels, k)
    assert np.array_equal(counts.read(), wc)
    assert np.array_equal(bits(sums.read()), bits(ws))
    # An empty selection zeroes the sums and counts.
    engine.scatter_add(xb, d, None, range(5, 5), lab, k, sums, counts)
    assert not sums.read().any() and not counts.read().any()


def test_scatter_add_bad_label_is_an_error(engine):
    d, k = 8, 4
    xb = engine.bind(np.ones((10, d), np.float32), d)
    lab = engine.upload_u32(np.array([0, 1, 2, 3, 4, 0, 1, 2, 3, 0], np.uint32))
    sums, counts = engine.zeros_f32(k * d), engine.zeros_u32(k)
    engine.scatter_add(xb, d, None, range(0, 10), lab, k, sums, counts)
    with pytest.raises(eb.EngineError) as ei:
        engine.sync()
    assert ei.value.code == eb.INVALID_ARGUMENT and "label" in str(ei.value)
    engine.sync()  # the error was reported once; the engine stays usable


@pytest.mark.parametrize("d,k", [(768, 64), (13, 70), (20, 300), (64, 1), (768, 1024)])
def test_ema_bit_equal(engine, d, k):
    x = mixture(max(k, 16), d, 7, 0.5, False, 3 * d + k)
    rng = np.random.default_rng(k)
    counts = rng.integers(0, 5, k).astype(np.uint32)
    sums = (x[:k] * np.float32(3.0)).ravel()
    pos0 = x[:k].ravel()
    for alpha, u0 in [(0.37, 0.8), (1.0, 0.5), (0.9, 0.0), (0.7281826767210002, 1.5e-5)]:
        usage0 = (np.float32(u0) + (np.arange(k) % 5).astype(np.float32) * np.float32(0.125))
        p, u = engine.upload_f32(pos0), engine.upload_f32(usage0)
        s, c = engine.upload_f32(sums), engine.upload_u32(counts)
        engine.ema_update(p, u, s, c, k, d, alpha)
        wp, wu = oracle.ema_update(pos0, usage0, sums, counts, k, d, alpha)
        assert np.array_equal(bits(p.read()), bits(wp))
        assert np.array_equal(bits(u.read()), bits(wu))


@pytest.mark.parametrize("d,k", [(768, 64), (13, 70), (20, 300), (768, 1024)])
def test_split_bit_equal(engine, d, k):
    x = mixture(k, d, 7, 0.5, False, d + k)
    pos = x.ravel().copy()
    pos[d:2 * d] = 0.0  # a zero donor: the child-nudge path
    pos[2 * d:3 * d] = np.float32(3.4e38)  # overflow: nudged down
    usage = (1.0 + np.arange(k) * 0.37).astype(np.float32)
    plan = [(j, k - 1 - j) for j in range(k // 2) if j % 3 != 2 and j != k - 1 - j]
    p, u = engine.upload_f32(pos), engine.upload_f32(usage)
    engine.split(p, u, plan, d)
    wp, wu = oracle.split(pos, usage, d, plan)
    assert np.array_equal(bits(p.read()), bits(wp))
    assert np.array_equal(bits(u.read()), bits(wu))


def test_split_rejects_overlapping_plans(engine):
    d, k = 4, 6
    p, u = engine.zeros_f32(k * d), engine.zeros_f32(k)
    with pytest.raises(eb.EngineError) as ei:
        engine.split(p, u, [(0, 5), (0, 4)], d)
    assert ei.value.code == eb.INVALID_ARGUMENT
    with pytest.raises(eb.EngineError):
        engine.split(p, u, [(0, 6)], d)


@pytest.mark.parametrize("n,d", [(1000, 768), (513, 13), (2000, 20), (300, 64), (77, 1)])
def test_norms_and_normalize_bit_equal(engine, n, d):
    m = mixture(n, d, 7, 0.5, False, n + d)
    rows = min(n, 1100)
    m = m[:rows].copy()
    m[0] = 0.0
    if rows > 1:
        m[1] *= np.float32(1e30)
    mb = engine.upload_f32(m)
    nb = engine.zeros_f32(rows)
    engine.row_norms(mb, rows, d, nb)
    assert np.array_equal(bits(nb.read()), bits(oracle.row_norms(m.ravel(), d)))
    ub = engine.zeros_f32(rows * d)
    engine.normalize_rows(mb, rows, d, ub)
    assert np.array_equal(bits(ub.read()), bits(oracle.normalize_rows(m.ravel(), d)))


def test_host_copies_large_pageable_and_pinned(engine):
    """Uploads, writes and reads of host arrays from 1 MB up (the staged path
    for pageable memory: two pinned buffers of 32 MB, several chunks, odd
    offsets and lengths) and of pinned arrays return the bytes unchanged."""
    import torch

    rng = np.random.default_rng(12)
    n = 70 * 1024 * 1024 // 4 + 13  # 70 MB and a ragged tail: three staging chunks
    v = rng.standard_normal(n).astype(np.float32)
    b = engine.upload_f32(v)
    assert np.array_equal(b.read().view(np.uint32), v.view(np.uint32))
    lo, hi = 1_000_003, n - 777
    assert np.array_equal(b.read(lo, hi).view(np.uint32), v[lo:hi].view(np.uint32))
    w = rng.standard_normal(9_000_001).astype(np.float32)
    b.write(123_457, w)
    v[123_457:123_457 + w.size] = w
    assert np.array_equal(b.read().view(np.uint32), v.view(np.uint32))
    pv = torch.from_numpy(v.copy()).pin_memory()
    b2 = engine.upload_f32(pv.numpy())
    assert np.array_equal(b2.read().view(np.uint32), v.view(np.uint32))
    b.free()
    b2.free()
