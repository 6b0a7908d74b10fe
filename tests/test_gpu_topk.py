"""kNN top-k on the B200 against the oracle: ids and scores bit-equal.

The exact oracle scores every pair with the FMA chain and orders by (score
desc, id asc) (crates/emeans-core/src/knn.rs:47-107); the shapes follow the
reference contract (crates/emeans-core/src/core/contract.rs:100-108,143-160):
small queries against data, a self-join with exclude_self, padding when there
are fewer rows than kk, and duplicate data rows (exact ties at rank 0). Each
shape runs on the exact SIMT kernel (screen mode 0) and on the tensor-core
screen in top-k mode (screen mode 2), and the kNN self-join config's shape
(unit rows with near-duplicates, kk 10) runs scaled down.
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, mixture

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[0, 2], ids=["exact", "screen"])
def eng(engine, request):
    """The session engine on the exact SIMT top-k (0) or the tcgen05 screen (2)."""
    engine.set_screen_mode(request.param)
    yield engine
    engine.set_screen_mode(1)


@pytest.mark.parametrize("m,n,d,kk", [(300, 300, 768, 16), (200, 900, 20, 5), (130, 7, 33, 10)])
def test_contract_shapes(eng, m, n, d, kk):
    data = mixture(n, d, 9, 0.3, True, m + n)
    q = mixture(m, d, 9, 0.3, True, m * 7 + n)
    gi, gs = eng.topk(q, data, d, kk)
    wi, ws = oracle.topk(q, data, d, kk)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
    if m == n:
        gi, gs = eng.topk(data, data, d, kk, exclude_self=True)
        wi, ws = oracle.topk(data, data, d, kk, exclude_self=True)
        assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))


def test_production_duplicates(eng):
    n, d = 16384, 768
    data = mixture(n, d, 9, 0.3, True, 77)
    data[8192:8192 + 512] = data[192:192 + 512]
    rows = [192 + i if i % 2 == 0 else (i * 61) % n for i in range(64)]
    q = data[rows]
    gi, gs = eng.topk(q, data, d, 16)
    wi, ws = oracle.topk(q, data, d, 16)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
    # The duplicate with the lower id ranks first.
    gi = gi.reshape(64, 16)
    for i in range(0, 64, 2):
        assert gi[i, 0] == 192 + i and gi[i, 1] == 8192 + i


def test_self_join_with_padding(eng):
    d = 12
    data = np.random.default_rng(3).standard_normal((5, d)).astype(np.float32)
    gi, gs = eng.topk(data, data, d, 8, exclude_self=True)
    gi, gs = gi.reshape(5, 8), gs.reshape(5, 8)
    assert np.all(gi[:, 4:] == 0xFFFFFFFF) and np.all(gs[:, 4:] == -np.inf)
    for i in range(5):
        assert i not in gi[i, :4]


def test_knn_self_helper(eng):
    data = mixture(500, 64, 20, 0.2, True, 5)
    ids, sims = eb.knn_self(data, 64, 10, engine=eng)
    wi, ws = oracle.topk(data, data, 64, 10, exclude_self=True)
    assert np.array_equal(ids.ravel(), wi) and np.array_equal(bits(sims.ravel()), bits(ws))
    with pytest.raises(ValueError):
        eb.knn_self(data, 64, 17, engine=eng)


def test_self_join_config_shape(engine):
    """The kNN self-join config's rows, scaled: unit rows from a mixture
    (sigma 0.4) with 5% near-duplicates (a row plus N(0, 0.01^2), normalised),
    inner product, kk 10, self excluded; auto mode takes the screen."""
    engine.set_screen_mode(1)
    n, d, kk = 6000, 384, 10
    rng = np.random.default_rng(4)
    means = rng.standard_normal((200, d)).astype(np.float32)
    x = means[rng.integers(0, 200, n)] + np.float32(0.4) * rng.standard_normal((n, d),
                                                                               dtype=np.float32)
    dup = rng.choice(n, n // 20, replace=False)
    src = rng.integers(0, n, n // 20)
    x[dup] = x[src] + np.float32(0.01) * rng.standard_normal((n // 20, d), dtype=np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    x = x.astype(np.float32)
    s0 = engine.stats()
    gi, gs = engine.topk(x, x, d, kk, exclude_self=True)
    s1 = engine.stats()
    wi, ws = oracle.topk(x, x, d, kk, exclude_self=True)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
    assert s1["screened_rows"] - s0["screened_rows"] == n


@pytest.mark.parametrize("case", ["scaled", "zero_rows", "nonfinite_queries", "nonfinite_data"])
def test_edge_values(eng, case):
    """Rows whose norms span six decades (the screen gives the database rows
    one scale, so small rows keep few digits and their windows widen), zero
    rows, and non-finite values in queries or data (rows the screen cannot
    certify go to the exact scan): ids and scores equal to the oracle's."""
    m, n, d, kk = 300, 2000, 100, 8
    rng = np.random.default_rng(11)
    data = mixture(n, d, 9, 0.5, False, 31)
    q = mixture(m, d, 9, 0.5, False, 32)
    if case == "scaled":
        data *= (10.0 ** rng.uniform(-3, 3, n)).astype(np.float32)[:, None]
        q *= (10.0 ** rng.uniform(-3, 3, m)).astype(np.float32)[:, None]
    elif case == "zero_rows":
        q[7] = 0.0
        data[[11, 12, 500]] = 0.0
    elif case == "nonfinite_queries":
        q[5, 3] = np.nan
        q[17, 0] = np.inf
        q[100] = -np.inf
    else:
        data[40, 2] = np.nan
    gi, gs = eng.topk(q, data, d, kk)
    wi, ws = oracle.topk(q, data, d, kk)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
