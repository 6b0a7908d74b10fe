"""Generate the golden vectors that pin the CPU oracle (tests/golden/golden.json).

Runs the reference's own Python implementation of e-means (the vendored faiss
``contrib/e_means`` package, ``reference/faiss_e_means`` inside the reference
checkout) in this container. faiss itself is not installed here: the one call
the package makes into it, ``faiss.knn`` (e_means.py:302-309), is replaced by
an exhaustive numpy search with the same outputs (sorted distances or inner
products and their ids).

Writes:
  golden.json    recipes, cosine alphas, MT19937 streams, training runs, and
                 exact FMA-chain dot products computed with rational arithmetic
  g_e8.f32, g_s24.f32   the seeded training inputs of the runs

Usage: python tests/golden/make_golden.py [/path/to/reference]
The reference checkout is the first argument, or $EMEANS_REFERENCE.
"""

from __future__ import annotations

import json
import os
import pathlib
import sys
import types
from fractions import Fraction

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def faiss_standin() -> types.ModuleType:
    """numpy stand-in for the single faiss entry point e_means.py uses."""
    mod = types.ModuleType("faiss")
    mod.METRIC_INNER_PRODUCT = 0
    mod.METRIC_L2 = 1

    def knn(xq, xb, k, metric=1):
        xq = np.ascontiguousarray(xq, dtype=np.float32)
        xb = np.ascontiguousarray(xb, dtype=np.float32)
        ip = xq @ xb.T
        if metric == mod.METRIC_INNER_PRODUCT:
            order = np.argsort(-ip, axis=1, kind="stable")[:, :k]
            return np.take_along_axis(ip, order, 1), order.astype(np.int64)
        dist = (xq * xq).sum(1)[:, None] + (xb * xb).sum(1)[None, :] - 2 * ip
        dist = np.maximum(dist, 0)
        order = np.argsort(dist, axis=1, kind="stable")[:, :k]
        return np.take_along_axis(dist, order, 1), order.astype(np.int64)

    mod.knn = knn
    return mod


def f32_round(q: Fraction) -> np.float32:
    """Round a rational to the nearest float32, ties to even (no double rounding)."""
    f = np.float32(float(q))
    best = f
    for g in (np.nextafter(f, np.float32(-np.inf)), np.nextafter(f, np.float32(np.inf))):
        eg, eb = abs(Fraction(float(g)) - q), abs(Fraction(float(best)) - q)
        if eg < eb or (eg == eb and (int(g.view(np.uint32)) & 1) == 0):
            best = g
    return np.float32(best)


def fma_chain(x: np.ndarray, c: np.ndarray) -> np.float32:
    """acc = 0; acc = fma(x_t, c_t, acc) for t in order, exactly (assign/fused.rs:12-16)."""
    acc = np.float32(0.0)
    for a, b in zip(x.tolist(), c.tolist()):
        acc = f32_round(Fraction(a) * Fraction(b) + Fraction(float(acc)))
    return acc


def tiny(n, d, centers, spherical, seed):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((centers, d)).astype(np.float32) * 3
    x = c[rng.integers(0, centers, n)] + rng.standard_normal((n, d)).astype(np.float32)
    if spherical:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype("<f4")


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EMEANS_REFERENCE")
    if not src:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set EMEANS_REFERENCE)")
    ref = pathlib.Path(src)
    sys.modules["faiss"] = faiss_standin()
    sys.path.insert(0, str(ref / "reference"))
    from faiss_e_means import NumpyEmeans  # noqa: E402
    from faiss_e_means.base import (  # noqa: E402
        _epoch_rows, _epoch_seed, _resolve_batch_law, _resolve_recipe,
        _resolve_unused_threshold, _scheduled_alpha,
    )

    recipes = []
    for n in [1_000, 20_000, 200_000, 33, 999_999]:
        for k in [8, 32, 1024, 65536]:
            for nepochs in [1, 2.5, 5, 0.4]:
                for law in ["auto", "throughput", "quality"]:
                    for d in [8, 64, 768]:
                        resolved, _ = _resolve_batch_law(law, d)
                        b, a0 = _resolve_recipe(n, k, nepochs, resolved, None, None)
                        rows = _epoch_rows(n, nepochs)
                        steps = [(r + b - 1) // b for r in rows]
                        recipes.append(dict(n=n, k=k, nepochs=nepochs, law=law, d=d,
                                            resolved=resolved, batch_size=b, alpha0=a0,
                                            epoch_rows=rows, epoch_steps=steps,
                                            unused_threshold=_resolve_unused_threshold(None, d)))
    for n, k, bs, a0 in [(20_000, 64, 1000, None), (50_000, 16, 99_999, None),
                         (200_000, 1024, 4096, 0.3)]:
        b, alpha = _resolve_recipe(n, k, 5, "throughput", bs, a0)
        recipes.append(dict(n=n, k=k, nepochs=5, law="given", d=64, given_batch_size=bs,
                            given_alpha0=a0, batch_size=b, alpha0=alpha))

    alphas = [dict(alpha0=a0, step=s, total=t, alpha=_scheduled_alpha(a0, s, t))
              for a0 in [0.83, 0.0123, 1.0] for t in [1, 13, 65, 100]
              for s in range(0, t + 2, max(1, t // 7))]

    mt = []
    for seed in [0, 7, 1234, _epoch_seed(7, 4), 2**32 - 1]:
        for n in [1, 3, 64, 20_000, 200_000]:
            perm = np.random.RandomState(seed).permutation(n)
            m = min(n, 5000)
            mt.append(dict(seed=seed, n=n, head=perm[:48].tolist(),
                           tail=perm[-16:].tolist(),
                           sum=int(perm[:m].astype(np.int64) @ np.arange(m))))
        mt.append(dict(seed=seed, random_sample=np.random.RandomState(seed)
                       .random_sample(10).tolist()))

    runs = []
    data = {"g_e8": tiny(1200, 8, 7, False, 23), "g_s24": tiny(900, 24, 5, True, 29)}
    for name, x in data.items():
        x.tofile(HERE / f"{name}.f32")
    for name, k, nepochs, law, spherical, seeds in [
        ("g_e8", 10, 3, "auto", False, [1234, 11]),
        ("g_s24", 9, 2.5, "throughput", True, [1234, 5]),
        ("g_e8", 33, 1.5, "quality", False, [3]),
    ]:
        x = data[name]
        n, d = x.shape
        for seed in seeds:
            m = NumpyEmeans(d, k, nepochs=nepochs, batch_law=law, seed=seed,
                            spherical=spherical)
            cent, labels = m.train(x)
            score, alabels = m.assign(x)
            runs.append(dict(
                data=name, n=n, d=d, k=k, nepochs=nepochs, batch_law=law, seed=seed,
                spherical=spherical, batch_size=m.recipe["batch_size"],
                alpha0=m.recipe["alpha0"],
                obj=[float(s["obj"]) for s in m.iteration_stats],
                imbalance=[float(s["imbalance_factor"]) for s in m.iteration_stats],
                nsplit=[int(s["nsplit"]) for s in m.iteration_stats],
                centroids=[float(v) for v in np.asarray(cent).ravel()],
                labels=[int(v) for v in labels],
                assign_labels=[int(v) for v in alabels],
                assign_scores=[float(v) for v in score],
            ))

    # Exact single-rounding FMA chains (known answers for the top-1 float order).
    rng = np.random.default_rng(5)
    chains = []
    for d in [1, 7, 64, 130]:
        xs = (rng.standard_normal((3, d)) * rng.choice([1e-3, 1, 1e3], (3, 1))).astype(np.float32)
        cs = rng.standard_normal((4, d)).astype(np.float32)
        for i in range(3):
            for j in range(4):
                chains.append(dict(x=[float(v) for v in xs[i]], c=[float(v) for v in cs[j]],
                                   dot=float(fma_chain(xs[i], cs[j]))))

    out = HERE / "golden.json"
    out.write_text(json.dumps(dict(recipes=recipes, alphas=alphas, mt19937=mt, runs=runs,
                                   fma_chains=chains), separators=(",", ":")))
    print(out, len(recipes), len(alphas), len(mt), len(runs), len(chains),
          [r["nsplit"] for r in runs])


if __name__ == "__main__":
    main()
