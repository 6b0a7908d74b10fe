"""kNN top-k on the B200 against the oracle: ids and scores bit-equal.

The exact oracle scores every pair with the FMA chain and orders by (score
desc, id asc) (crates/emeans-core/src/knn.rs:47-107); the shapes follow the
reference contract (crates/emeans-core/src/core/contract.rs:100-108,143-160):
small queries against data, a self-join with exclude_self, padding when there
are fewer rows than kk, and duplicate data rows (exact ties at rank 0).
"""

import numpy as np
import pytest

import emeans_b200 as eb
import oracle
from tests.helpers import bits, mixture

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,d,kk", [(300, 300, 768, 16), (200, 900, 20, 5), (130, 7, 33, 10)])
def test_contract_shapes(engine, m, n, d, kk):
    data = mixture(n, d, 9, 0.3, True, m + n)
    q = mixture(m, d, 9, 0.3, True, m * 7 + n)
    gi, gs = engine.topk(q, data, d, kk)
    wi, ws = oracle.topk(q, data, d, kk)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
    if m == n:
        gi, gs = engine.topk(data, data, d, kk, exclude_self=True)
        wi, ws = oracle.topk(data, data, d, kk, exclude_self=True)
        assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))


def test_production_duplicates(engine):
    n, d = 16384, 768
    data = mixture(n, d, 9, 0.3, True, 77)
    data[8192:8192 + 512] = data[192:192 + 512]
    rows = [192 + i if i % 2 == 0 else (i * 61) % n for i in range(64)]
    q = data[rows]
    gi, gs = engine.topk(q, data, d, 16)
    wi, ws = oracle.topk(q, data, d, 16)
    assert np.array_equal(gi, wi) and np.array_equal(bits(gs), bits(ws))
    # The duplicate with the lower id ranks first.
    gi = gi.reshape(64, 16)
    for i in range(0, 64, 2):
        assert gi[i, 0] == 192 + i and gi[i, 1] == 8192 + i


def test_self_join_with_padding(engine):
    d = 12
    data = np.random.default_rng(3).standard_normal((5, d)).astype(np.float32)
    gi, gs = engine.topk(data, data, d, 8, exclude_self=True)
    gi, gs = gi.reshape(5, 8), gs.reshape(5, 8)
    assert np.all(gi[:, 4:] == 0xFFFFFFFF) and np.all(gs[:, 4:] == -np.inf)
    for i in range(5):
        assert i not in gi[i, :4]


def test_knn_self_helper(engine):
    data = mixture(500, 64, 20, 0.2, True, 5)
    ids, sims = eb.knn_self(data, 64, 10, engine=engine)
    wi, ws = oracle.topk(data, data, 64, 10, exclude_self=True)
    assert np.array_equal(ids.ravel(), wi) and np.array_equal(bits(sims.ravel()), bits(ws))
    with pytest.raises(ValueError):
        eb.knn_self(data, 64, 17, engine=engine)
