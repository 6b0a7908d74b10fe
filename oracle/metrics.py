"""CPU restatement of the reference's internal clustering scores (test
infrastructure only: imported by tests/ and bench.py's CPU-baseline leg).

Follows crates/emeans-cluster/src/metrics.rs:115-274 step by step in numpy
f64: cluster sums in row order (np.add.at applies in index order), sums of
squares and totals as sequential sums (the last element of a cumulative sum),
and the per-row, per-cluster and final formulas in the reference's operation
order. The n x k_eff product is an f32 matrix product, as the reference's
gemm_nt (crates/emeans-core/src/assign.rs:813-825) is; its addition order is
the BLAS library's, so this restatement agrees with the reference to rounding.

Pinned against scikit-learn's silhouette (cosine), Calinski-Harabasz and
Davies-Bouldin scores on the fixtures tests/golden/make_metrics_golden.py
writes, to the reference test's own tolerance (crates/emeans-cluster/tests/
metrics.rs: relative 1e-5).
"""

from __future__ import annotations

import numpy as np


def _seq(a, axis=-1):
    """Sequential (left-to-right) sum along axis."""
    a = np.asarray(a, np.float64)
    if a.shape[axis] == 0:
        return np.zeros(np.delete(a.shape, axis)) if a.ndim > 1 else 0.0
    return np.take(np.cumsum(a, axis=axis), -1, axis=axis)


def internal_scores(x, d, labels, k):
    x = np.asarray(x, np.float32).reshape(-1, d)
    labels = np.asarray(labels, np.int64).ravel()
    n = x.shape[0]
    if labels.size != n:
        raise ValueError("one label per row")
    if n and labels.max() >= k:
        raise ValueError("label out of range")
    sizes = np.bincount(labels, minlength=k).astype(np.int64)
    sums = np.zeros((k, d), np.float64)
    np.add.at(sums, labels, x.astype(np.float64))  # metrics.rs:127-134, row order
    live = np.flatnonzero(sizes > 0)
    k_eff = live.size
    out = {"k_eff": int(k_eff), "sizes": sizes}
    if n == 0:
        out.update(silhouette=0.0, calinski_harabasz=0.0, davies_bouldin=0.0, objective=0.0)
        return out
    sums32 = sums[live].astype(np.float32)
    sq_sum = _seq(sums[live] * sums[live], axis=1)            # metrics.rs:141-144
    slot = np.zeros(k, np.int64)
    slot[live] = np.arange(k_eff)
    x64 = x.astype(np.float64)
    xx = _seq(x64 * x64, axis=1)                              # metrics.rs:149-152

    g = (x @ sums32.T).astype(np.float32)                     # gemm_nt, metrics.rs:163
    own = slot[labels]
    na = sizes[live][own].astype(np.float64)
    dot_own = g[np.arange(n), own].astype(np.float64)
    dist = np.sqrt(np.maximum(xx - 2.0 * dot_own / na + sq_sum[own] / (na * na), 0.0))
    cos_c = dot_own / np.maximum(np.sqrt(sq_sum[own]), 1e-30)
    obj = 2.0 - 2.0 * cos_c
    q = g.astype(np.float64) / sizes[live].astype(np.float64)[None, :]
    q[np.arange(n), own] = -np.inf
    b = (1.0 - q).min(axis=1) if k_eff >= 2 else np.full(n, np.inf)
    a = 1.0 - (dot_own - xx) / (na - 1.0)
    m = np.maximum(a, b)
    with np.errstate(divide="ignore", invalid="ignore"):
        sil = np.where(m > 0.0, (b - a) / m, 0.0)
    sil = np.where((k_eff < 2) | (na < 2.0), 0.0, sil)
    scatter = np.zeros(k_eff, np.float64)
    np.add.at(scatter, own, dist)                             # metrics.rs:182-184
    nf = float(max(n, 1))

    total_xx = _seq(xx)                                       # metrics.rs:189-216
    within = total_xx - _seq(sq_sum / sizes[live])
    grand = np.zeros(d, np.float64)
    for j in live:
        grand += sums[j]
    total = total_xx - _seq(grand * grand) / nf
    between = total - within
    if k_eff < 2 or n <= k_eff or within <= 0.0:
        ch = 0.0
    else:
        ch = (between / (k_eff - 1)) / (within / (n - k_eff))

    db = 0.0                                                  # metrics.rs:217-256
    if k_eff >= 2:
        means = sums[live] / sizes[live][:, None].astype(np.float64)
        spread = scatter / sizes[live]
        worst = np.zeros(k_eff)
        for ai in range(k_eff):
            diff = means[ai][None, :] - means
            mdist = np.sqrt(_seq(diff * diff, axis=1))
            with np.errstate(divide="ignore"):
                v = np.where(mdist > 0.0, (spread[ai] + spread) / mdist, np.inf)
            v[ai] = 0.0
            worst[ai] = max(0.0, float(v.max()))
        db = _seq(worst) / k_eff

    out.update(silhouette=_seq(sil) / nf, calinski_harabasz=float(ch),
               davies_bouldin=float(db), objective=_seq(obj) / nf)
    return out
