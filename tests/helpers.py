"""Deterministic inputs for the parity tests.

``mixture`` follows the reference contract suite's generator
(crates/emeans-core/src/core/contract.rs:40-60): Box-Muller normals from the
MT19937 ``random_sample`` stream (numpy's legacy RandomState is the same
stream), ``centers`` Gaussian means, rows = mean[i % centers] + sigma * noise,
optionally unit-normalised, cast to f32.
"""

from __future__ import annotations

import numpy as np


def mixture(n, d, centers, sigma, unit, seed):
    rs = np.random.RandomState(seed)
    total = centers * d + n * d
    s = rs.random_sample(2 * total)
    u1 = np.maximum(s[0::2], 1e-300)
    u2 = s[1::2]
    g = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    cs = g[: centers * d].reshape(centers, d)
    noise = g[centers * d:].reshape(n, d)
    rows = cs[np.arange(n) % centers] + sigma * noise
    if unit:
        rows = rows / np.maximum(np.sqrt((rows * rows).sum(1, keepdims=True)), 1e-12)
    return rows.astype(np.float32)


def contract_centroids(x, d, k):
    """check(): centroids = the first rows, cycled, times 0.95 (contract.rs:93-98)."""
    n = x.shape[0]
    flat = x[: min(k, n)].ravel()
    reps = -(-(k * d) // flat.size)
    return (np.tile(flat, reps)[: k * d] * np.float32(0.95)).astype(np.float32).reshape(k, d)


def production_centroids(x, k):
    """check_production(): the last 256 centroids copy earlier ones (contract.rs:128-141)."""
    n, d = x.shape
    base = k - 256
    c = np.zeros((k, d), np.float32)
    for j in range(k):
        if j < base:
            c[j] = x[(j * 37) % n] * np.float32(0.95)
        else:
            c[j] = c[(j * 7) % base]
    return c


def near_tie_centroids(d, k, seed):
    """Adversarial near-ties: groups of 32 centroids within 1e-6 of one another,
    exact duplicate pairs, and centroids scaled by 1e3 / 1e-3 (the shape of the
    reference's CUDA near-tie suite, crates/emeans-cuda/tests/contract.rs:45-152)."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal((k // 32 + 1, d)).astype(np.float32)
    base /= np.linalg.norm(base, axis=1, keepdims=True)
    c = np.empty((k, d), np.float32)
    for j in range(k):
        g = base[j // 32]
        c[j] = g + np.float32(1e-6) * rng.standard_normal(d).astype(np.float32)
    for j in range(0, k - 1, 7):
        c[j + 1] = c[j]
    return c


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)
