"""Empty inputs on the B200, as the reference contract treats them.

An empty selection writes nothing (outputs outside the selection stay
untouched: crates/emeans-core/src/core/contract.rs:225-231); an assign of
zero rows returns empty labels and scores; a top-k over zero queries returns
nothing, and one over zero data rows is refused as the reference's CUDA
Device::topk refuses it (crates/emeans-cuda/src/lib.rs:1246, "no data rows";
the reference CPU search, crates/emeans-core/src/knn.rs:53-107, pads every
list instead). Each case runs on the
exact SIMT kernels (screen mode 0) and with the tensor-core screen allowed
(screen mode 2), and is checked against the oracle where it has an output.
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, mixture

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[0, 2], ids=["exact", "screen"])
def eng(engine, request):
    engine.set_screen_mode(request.param)
    yield engine
    engine.set_screen_mode(1)


@pytest.mark.parametrize("metric", [eb.L2, eb.IP])
def test_top1_empty_selection_leaves_outputs(eng, metric):
    n, d, k = 600, 64, 300
    x = mixture(n, d, 9, 0.4, False, 5)
    c = x[::2][:k].copy()
    xb = eng.bind(x, d)
    cb = eng.upload_f32(c)
    cn = eng.upload_f32(oracle.row_norms(c.ravel(), d)) if metric == eb.L2 else None
    lab = eng.upload_u32(np.full(n, 7, np.uint32))
    sco = eng.upload_f32(np.full(n, 2.5, np.float32))
    eng.top1(xb, d, None, range(300, 300), cb, cn, k, metric, lab, sco)
    assert np.all(lab.read() == 7) and np.all(sco.read() == np.float32(2.5))
    # A non-empty selection after it still matches the oracle.
    eng.top1(xb, d, None, range(100, 400), cb, cn, k, metric, lab, sco)
    wl, ws = oracle.top1(x[100:400].ravel(), d, c.ravel(), metric)
    gl, gs = lab.read(), sco.read()
    assert np.array_equal(gl[100:400], wl) and np.array_equal(bits(gs[100:400]), bits(ws))
    assert np.all(gl[:100] == 7) and np.all(gl[400:] == 7)


def test_assign_zero_rows(eng):
    d, k = 32, 40
    c = mixture(k, d, 4, 0.3, True, 9)
    labels, scores = eng.assign(np.zeros((0, d), np.float32), d, c, eb.IP)
    assert labels.size == 0 and scores.size == 0


def test_topk_zero_queries_and_zero_data(eng):
    d, kk = 48, 6
    data = mixture(500, d, 9, 0.3, True, 3)
    q = mixture(20, d, 9, 0.3, True, 4)
    gi, gs = eng.topk(np.zeros((0, d), np.float32), data, d, kk)
    assert gi.size == 0 and gs.size == 0
    with pytest.raises(eb.EngineError) as err:
        eng.topk(q, np.zeros((0, d), np.float32), d, kk)
    assert err.value.code == eb.INVALID_ARGUMENT and "no data rows" in str(err.value)
    # The engine is still usable.
    gi, gs = eng.topk(q, data, d, kk)
    wi, ws = oracle.topk(q, data, d, kk)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
