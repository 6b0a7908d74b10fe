"""Writes tests/golden/metrics.json and metrics_<name>.f32: seeded unit-row
data sets with labellings, and scikit-learn's silhouette (cosine distance),
Calinski-Harabasz and Davies-Bouldin scores of each, the values the
reference's metrics test checks its internal scores against (to relative
1e-5). Run: python tests/golden/make_metrics_golden.py
"""
import json
import os

import numpy as np
from sklearn.metrics import calinski_harabasz_score, davies_bouldin_score, silhouette_score

HERE = os.path.dirname(os.path.abspath(__file__))


def unit(a):
    a = a.astype(np.float32)
    return (a / np.linalg.norm(a, axis=1, keepdims=True)).astype(np.float32)


def blobs(rng, n, d, k, sigma):
    centers = rng.standard_normal((k, d))
    lab = rng.integers(0, k, n)
    return unit(centers[lab] + sigma * rng.standard_normal((n, d))), lab


def cases():
    rng = np.random.default_rng(2024)
    x, lab = blobs(rng, 300, 8, 3, 0.3)
    yield "blobs3", x, lab, 3
    # Labels from a noisier truth, a never-used label and a three-row cluster.
    # (No singleton: the reference's distance to a one-row cluster's mean is
    # sqrt of a cancellation of f32-rounded products, not 0 as scikit-learn's.)
    x, lab = blobs(rng, 2000, 32, 10, 0.8)
    lab = lab.copy()
    lab[lab == 7] = 3          # label 7 empty
    lab[5:8] = 11              # label 11: three rows
    yield "sparse_labels", x, lab, 12
    # Many small clusters, d not a multiple of 4.
    x, lab = blobs(rng, 1500, 30, 40, 0.5)
    yield "k40_d30", x, lab, 40


def main():
    out = {"cases": []}
    for name, x, lab, k in cases():
        x64 = x.astype(np.float64)
        out["cases"].append({
            "name": name, "n": int(x.shape[0]), "d": int(x.shape[1]), "k": int(k),
            "labels": [int(v) for v in lab],
            "silhouette": float(silhouette_score(x64, lab, metric="cosine")),
            "calinski_harabasz": float(calinski_harabasz_score(x64, lab)),
            "davies_bouldin": float(davies_bouldin_score(x64, lab)),
        })
        x.astype("<f4").tofile(os.path.join(HERE, f"metrics_{name}.f32"))
    with open(os.path.join(HERE, "metrics.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
