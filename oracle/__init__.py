"""ctypes loader for the CPU oracle (test infrastructure only).

The oracle restates the reference CPU path's float order (crate emeans-core)
in C++ (oracle.cpp). Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg may import this package; the product (``emeans_b200``) never
does.
"""

from __future__ import annotations

import ctypes as C
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

L2, IP = 0, 1
LAW = {"auto": 0, "throughput": 1, "quality": 2}

_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so with the Makefile next to this file."""
    src = os.path.join(HERE, "oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
        os.path.getmtime(src), os.path.getmtime(os.path.join(HERE, "oracle.h"))
    ):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return LIB_PATH


class RecipeT(C.Structure):
    _fields_ = [
        ("batch_size", C.c_int64),
        ("alpha0", C.c_double),
        ("resolved_law", C.c_int32),
        ("n_epochs", C.c_int32),
        ("steps_per_pass", C.c_int64),
        ("total_steps", C.c_int64),
        ("epoch_rows", C.c_int64 * 64),
        ("epoch_steps", C.c_int64 * 64),
    ]


class TrainCfg(C.Structure):
    _fields_ = [
        ("nepochs", C.c_double),
        ("batch_law", C.c_int32),
        ("spherical", C.c_int32),
        ("batch_size", C.c_int64),
        ("alpha0", C.c_double),
        ("unused_threshold", C.c_double),
        ("seed", C.c_uint32),
        ("capture", C.c_int32),
        ("chunk", C.c_int64),
        ("threads", C.c_int32),
    ]


class TrainOut(C.Structure):
    _fields_ = [
        ("centroids", C.POINTER(C.c_float)),
        ("positions", C.POINTER(C.c_float)),
        ("usage", C.POINTER(C.c_float)),
        ("labels", C.POINTER(C.c_int32)),
        ("obj", C.c_double * 64),
        ("imbalance", C.c_double * 64),
        ("nsplit", C.c_int64 * 64),
        ("n_epochs", C.c_int32),
        ("n_splits", C.c_int64),
        ("batch_size", C.c_int64),
        ("alpha0", C.c_double),
    ]


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _lib.orc_last_error.restype = C.c_char_p
        _lib.orc_scheduled_alpha.restype = C.c_double
        _lib.orc_scheduled_alpha.argtypes = [C.c_double, C.c_size_t, C.c_size_t]
        _lib.orc_unused_threshold.restype = C.c_double
        _lib.orc_unused_threshold.argtypes = [C.c_double, C.c_size_t]
        _lib.orc_epoch_seed.restype = C.c_uint32
        _lib.orc_epoch_seed.argtypes = [C.c_uint32, C.c_size_t]
        _lib.orc_numpy_sum_f32.restype = C.c_float
        _lib.orc_rng_new.restype = C.c_void_p
        _lib.orc_rng_new.argtypes = [C.c_uint32]
        _lib.orc_rng_free.argtypes = [C.c_void_p]
        _lib.orc_plan_revival.restype = C.c_size_t
        _lib.orc_plan_revival.argtypes = [C.c_void_p, C.c_size_t, C.c_double, C.c_void_p, C.c_void_p]
        _lib.orc_recipe.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, C.c_int,
                                    C.c_size_t, C.c_double, C.POINTER(RecipeT)]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _check(rc):
    if rc != 0:
        raise ValueError(lib().orc_last_error().decode())


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def permutation(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().orc_permutation(C.c_uint32(seed), C.c_size_t(n), _p(out))
    return out


def random_sample(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float64)
    lib().orc_random_sample(C.c_uint32(seed), C.c_size_t(count), _p(out))
    return out


def recipe(n, k, d, nepochs, law="auto", batch_size=None, alpha0=None) -> dict:
    r = RecipeT()
    _check(lib().orc_recipe(n, k, d, float(nepochs), LAW[law], batch_size or 0,
                            math.nan if alpha0 is None else float(alpha0), C.byref(r)))
    ne = r.n_epochs
    return dict(batch_size=r.batch_size, alpha0=r.alpha0, resolved_law=r.resolved_law,
                steps_per_pass=r.steps_per_pass, total_steps=r.total_steps,
                epoch_rows=list(r.epoch_rows[:ne]), epoch_steps=list(r.epoch_steps[:ne]))


def scheduled_alpha(alpha0, step, total):
    return lib().orc_scheduled_alpha(alpha0, step, total)


def unused_threshold(given, d):
    return lib().orc_unused_threshold(math.nan if given is None else given, d)


def epoch_seed(seed, epoch):
    return lib().orc_epoch_seed(seed, epoch)


def row_norms(m, d):
    m = f32(m)
    rows = m.size // d
    out = np.empty(rows, np.float32)
    lib().orc_row_norms(_p(m), C.c_size_t(rows), C.c_size_t(d), _p(out))
    return out


def normalize_rows(m, d):
    m = f32(m)
    out = np.empty_like(m)
    lib().orc_normalize_rows(_p(m), C.c_size_t(m.size // d), C.c_size_t(d), _p(out))
    return out


def top1(x, d, c, metric, ids=None, r0=0, r1=None, labels=None, scores=None, threads=None):
    """Labels and scores at positions r0..r1 (x[ids[p]] or x[p])."""
    x, c = f32(x), f32(c)
    n, k = x.size // d, c.size // d
    ids = None if ids is None else u32(ids)
    if r1 is None:
        r1 = len(ids) if ids is not None else n
    m = len(ids) if ids is not None else n
    labels = np.zeros(m, np.uint32) if labels is None else labels
    scores = np.zeros(m, np.float32) if scores is None else scores
    threads = threads or os.cpu_count() or 1
    _check(lib().orc_top1(_p(x), C.c_size_t(n), C.c_size_t(d), _p(ids), C.c_size_t(r0),
                          C.c_size_t(r1), _p(c), C.c_size_t(k), C.c_int(metric), _p(labels),
                          _p(scores), C.c_int(threads)))
    return labels, scores


def scatter_add(x, d, labels, k, ids=None, r0=0, r1=None, acc=None):
    x = f32(x)
    n = x.size // d
    labels = u32(labels)
    ids = None if ids is None else u32(ids)
    if r1 is None:
        r1 = len(labels)
    sums = np.empty(k * d, np.float32)
    counts = np.empty(k, np.uint32)
    _check(lib().orc_scatter_add(_p(x), C.c_size_t(n), C.c_size_t(d), _p(ids), C.c_size_t(r0),
                                 C.c_size_t(r1), _p(labels), C.c_size_t(k), _p(sums),
                                 _p(counts), _p(acc)))
    return sums, counts


def ema_update(pos, usage, sums, counts, k, d, alpha: float):
    """EmaStep::new(alpha) then the EMA step; returns new (pos, usage)."""
    pos, usage = f32(pos).copy(), f32(usage).copy()
    a32 = np.float32(alpha)
    decay = np.float32(1.0 - alpha)
    lib().orc_ema_update(_p(pos), _p(usage), _p(f32(sums)), _p(u32(counts)), C.c_size_t(k),
                         C.c_size_t(d), C.c_float(a32), C.c_float(decay), C.c_int(alpha == 1.0))
    return pos, usage


def split(pos, usage, d, pairs):
    pos, usage = f32(pos).copy(), f32(usage).copy()
    pairs = u32(np.asarray(pairs).reshape(-1))
    lib().orc_split(_p(pos), _p(usage), C.c_size_t(usage.size), C.c_size_t(d), _p(pairs),
                    C.c_size_t(pairs.size // 2))
    return pos, usage


def numpy_sum_f32(a):
    a = f32(a)
    return np.float32(lib().orc_numpy_sum_f32(_p(a), C.c_size_t(a.size)))


class Rng:
    """numpy legacy RandomState living across plan_revival calls."""

    def __init__(self, seed):
        self.h = lib().orc_rng_new(seed)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_rng_free(self.h)
            self.h = None

    def plan_revival(self, usage, tau):
        usage = f32(usage)
        out = np.empty(2 * usage.size, np.uint32)
        n = lib().orc_plan_revival(_p(usage), usage.size, tau, self.h, _p(out))
        return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


def closing_means(pos, sums, counts, k, d, spherical):
    out = np.empty(k * d, np.float32)
    lib().orc_closing_means(_p(f32(pos)), _p(f32(sums)),
                            _p(np.ascontiguousarray(counts, np.float64)), C.c_size_t(k),
                            C.c_size_t(d), C.c_int(int(spherical)), _p(out))
    return out


def topk(q, data, d, kk, exclude_self=False, threads=None):
    q, data = f32(q), f32(data)
    m, n = q.size // d, data.size // d
    ids = np.empty(m * kk, np.uint32)
    sims = np.empty(m * kk, np.float32)
    threads = threads or os.cpu_count() or 1
    _check(lib().orc_topk(_p(q), C.c_size_t(m), _p(data), C.c_size_t(n), C.c_size_t(d),
                          C.c_size_t(kk), C.c_int(int(exclude_self)), _p(ids), _p(sims),
                          C.c_int(threads)))
    return ids, sims


def topk_self_rows(data, d, q0, m, kk, threads=None):
    """The self-join's top-kk (self excluded) of the queries data[q0 .. q0 + m)
    against all of data."""
    data = f32(data)
    n = data.size // d
    ids = np.empty(m * kk, np.uint32)
    sims = np.empty(m * kk, np.float32)
    threads = threads or os.cpu_count() or 1
    _check(lib().orc_topk_self_rows(_p(data), C.c_size_t(n), C.c_size_t(d), C.c_size_t(q0),
                                    C.c_size_t(m), C.c_size_t(kk), _p(ids), _p(sims),
                                    C.c_int(threads)))
    return ids, sims


def train(x, d, k, nepochs=5.0, batch_law="auto", batch_size=None, alpha0=None, seed=1234,
          spherical=False, unused_threshold=None, chunk=None, init=None, state=None,
          threads=None):
    """The reference device loop on the oracle's ops (core/train.rs)."""
    x = f32(x)
    n = x.size // d
    cfg = TrainCfg(nepochs=float(nepochs), batch_law=LAW[batch_law], spherical=int(spherical),
                   batch_size=batch_size or 0,
                   alpha0=math.nan if alpha0 is None else float(alpha0),
                   unused_threshold=math.nan if unused_threshold is None else float(unused_threshold),
                   seed=seed, capture=1, chunk=chunk or 0,
                   threads=threads or os.cpu_count() or 1)
    cent = np.empty(k * d, np.float32)
    pos = np.empty(k * d, np.float32)
    usage = np.empty(k, np.float32)
    labels = np.empty(n, np.int32)
    out = TrainOut(centroids=cent.ctypes.data_as(C.POINTER(C.c_float)),
                   positions=pos.ctypes.data_as(C.POINTER(C.c_float)),
                   usage=usage.ctypes.data_as(C.POINTER(C.c_float)),
                   labels=labels.ctypes.data_as(C.POINTER(C.c_int32)))
    sp, su = (None, None) if state is None else (f32(state[0]), f32(state[1]))
    _check(lib().orc_train(_p(x), C.c_size_t(n), C.c_size_t(d), C.c_size_t(k), C.byref(cfg),
                           _p(None if init is None else f32(init)), _p(sp), _p(su),
                           C.byref(out)))
    ne = out.n_epochs
    return dict(centroids=cent, positions=pos, usage=usage, labels=labels,
                obj=list(out.obj[:ne]), imbalance=list(out.imbalance[:ne]),
                nsplit=list(out.nsplit[:ne]), n_splits=out.n_splits,
                batch_size=out.batch_size, alpha0=out.alpha0)
