"""emeans_b200: the emeans hot path on B200 (sm_100a), from Python.

A ctypes layer over libemeans_b200.so (the C ABI in include/emeans_b200.h).
It mirrors the reference's interfaces for this path:

- :class:`Engine` is the layer-1 op contract ``trait Device``
  (crates/emeans-core/src/core/mod.rs:71-178): buffers, ``top1``, ``topk``,
  ``scatter_add``, ``row_norms``, ``normalize_rows``, ``split``,
  ``ema_update``; plus ``train`` (``Engine::run_train``, the device loop of
  core/train.rs) and ``assign`` (``Assigner::assign``).
- :class:`B200Assigner` is ``trait Assigner`` (crates/emeans-core/src/assign.rs:71-117),
  the object ``make_assigner(Backend::Cuda)`` returns
  (crates/emeans-cluster/src/backend.rs:126-133).
- :func:`knn_self` / :func:`knn` follow crates/emeans-cluster/src/knn.rs:17-64.

There is no CPU fallback: without the built library or a B200 the calls
raise.
"""

from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

__all__ = ["Engine", "Buffer", "B200Assigner", "EngineError", "Config", "Trained",
           "DedupConfig", "DedupResult", "dedup", "dedup_with_neighbors",
           "knn", "knn_self", "L2", "IP", "lib_path", "load"]

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libemeans_b200.so"

L2, IP = 0, 1
F32, U32 = 0, 1
OK, INVALID_ARGUMENT, ERROR, INTERNAL = 0, 1, 2, 3
NONE_ID = 0xFFFFFFFF
GPU_KMAX = 16

_lib = None


class _Internal(C.Structure):
    """eb_internal (include/emeans_b200.h)."""
    _fields_ = [("k_eff", C.c_uint64), ("silhouette", C.c_double),
                ("calinski_harabasz", C.c_double), ("davies_bouldin", C.c_double),
                ("objective", C.c_double)]


class _DedupConfig(C.Structure):
    """eb_dedup_config (include/emeans_b200.h)."""
    _fields_ = [("k", C.c_size_t), ("sim_threshold", C.c_float), ("rep_threshold", C.c_float),
                ("max_gap_secs", C.c_double)]


class _DedupOut(C.Structure):
    """eb_dedup_out (include/emeans_b200.h)."""
    _fields_ = [("group_of", C.c_void_p), ("representatives", C.c_void_p),
                ("anchors", C.c_void_p), ("sizes", C.c_void_p), ("nn_sim", C.c_void_p),
                ("n_groups", C.c_uint64), ("linked_pairs", C.c_uint64),
                ("split_components", C.c_uint64)]


class EngineError(RuntimeError):
    """A non-OK status from the engine; ``code`` is the EB_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{ {1: 'INVALID_ARGUMENT', 2: 'ERROR', 3: 'INTERNAL'}.get(code, code)}] {msg}")
        self.code = code


class Stats(C.Structure):
    _fields_ = [("screened_rows", C.c_uint64), ("fallback_rows", C.c_uint64),
                ("rescored_candidates", C.c_uint64), ("exact_rows", C.c_uint64),
                ("kernel_launches", C.c_uint64), ("h2d_bytes", C.c_uint64)]


class TrainJob(C.Structure):
    _fields_ = [
        ("x", C.c_void_p), ("n", C.c_size_t), ("d", C.c_size_t), ("k", C.c_size_t),
        ("nepochs", C.c_double), ("batch_law", C.c_int32), ("spherical", C.c_int32),
        ("batch_size", C.c_int64), ("alpha0", C.c_double), ("unused_threshold", C.c_double),
        ("seed", C.c_uint32), ("capture", C.c_int32), ("chunk", C.c_int64),
        ("init", C.c_void_p), ("state_positions", C.c_void_p), ("state_usage", C.c_void_p),
        ("verbose", C.c_int32),
    ]


class TrainOut(C.Structure):
    _fields_ = [
        ("centroids", C.c_void_p), ("positions", C.c_void_p), ("usage", C.c_void_p),
        ("labels", C.c_void_p), ("obj", C.c_double * 64), ("imbalance", C.c_double * 64),
        ("nsplit", C.c_int64 * 64), ("epoch_time", C.c_double * 64), ("n_epochs", C.c_int32),
        ("n_splits", C.c_int64), ("batch_size", C.c_int64), ("alpha0", C.c_double),
        ("total_steps", C.c_int64),
    ]


def lib_path() -> str:
    return os.path.join(HERE, _LIB_NAME)


def load():
    """Load libemeans_b200.so; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m emeans_b200.build` "
                           "(nvcc, sm_100a); there is no CPU fallback")
    lib = C.CDLL(path)
    P, S, I = C.c_void_p, C.c_size_t, C.c_int
    sig = {
        "eb_last_error": (C.c_char_p, []),
        "eb_version": (C.c_char_p, []),
        "eb_engine_create": (I, [I, C.POINTER(P)]),
        "eb_engine_destroy": (I, [P]),
        "eb_engine_name": (I, [P, C.c_char_p, S]),
        "eb_flush": (I, [P]),
        "eb_sync": (I, [P]),
        "eb_get_stats": (I, [P, C.POINTER(Stats)]),
        "eb_engine_stream": (I, [P, C.POINTER(P)]),
        "eb_set_screen_mode": (I, [P, I]),
        "eb_buf_alloc": (I, [P, I, S, C.POINTER(P)]),
        "eb_buf_wrap": (I, [P, I, P, S, C.POINTER(P)]),
        "eb_buf_free": (I, [P, P]),
        "eb_buf_len": (S, [P]),
        "eb_buf_ptr": (P, [P]),
        "eb_buf_write": (I, [P, P, S, P, S]),
        "eb_buf_read": (I, [P, P, S, S, P]),
        "eb_buf_upload": (I, [P, I, P, S, C.POINTER(P)]),
        "eb_bind": (I, [P, P, S, S, C.POINTER(P)]),
        "eb_top1": (I, [P, P, S, P, S, S, P, P, S, I, P, P]),
        "eb_topk": (I, [P, P, S, P, S, S, S, I, P, P]),
        "eb_internal_scores": (I, [P, P, S, S, P, S, P, P]),
        "eb_scatter_add": (I, [P, P, S, P, S, S, P, S, P, P, P]),
        "eb_row_norms": (I, [P, P, S, S, P]),
        "eb_normalize_rows": (I, [P, P, S, S, P]),
        "eb_split": (I, [P, P, P, P, S, S]),
        "eb_ema_update": (I, [P, P, P, P, P, S, S, C.c_float, C.c_float, I]),
        "eb_bind_data": (I, [P, P, S, S]),
        "eb_unbind_data": (I, [P]),
        "eb_assign": (I, [P, P, S, S, P, S, P, S, I, P, P]),
        "eb_train": (I, [P, C.POINTER(TrainJob), C.POINTER(TrainOut)]),
        "eb_set_kernel_timing": (I, [P, I]),
        "eb_screen_timing": (I, [P, C.POINTER(C.c_double), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_uint64)]),
        "eb_topk_group": (I, [P, P, S, P, S, S, S, S, S, I, P, P]),
        "eb_group_unique_id": (I, [C.c_char_p]),
        "eb_engine_join": (I, [P, I, I, C.c_char_p]),
        "eb_engine_group": (I, [P, C.POINTER(I), C.POINTER(I)]),
        "eb_set_group_shard": (I, [P, I]),
        "eb_device_allocations": (I, [P, C.POINTER(C.c_uint64)]),
        "eb_group_allgather": (I, [P, P, S]),
        "eb_group_exchange": (I, [P, S, P]),
        "eb_group_exchange_info": (I, [P, P, P, S]),
        "eb_test_screen_dead_wait": (I, [P, I]),
        "eb_dedup_with_neighbors": (I, [P, S, S, P, P, S, P, P, P, C.POINTER(_DedupConfig),
                                        C.POINTER(_DedupOut)]),
        "eb_dedup": (I, [P, P, S, S, P, P, P, C.POINTER(_DedupConfig), C.POINTER(_DedupOut)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(rc: int):
    if rc != OK:
        raise EngineError(rc, load().eb_last_error().decode())


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


class Buffer:
    """An engine buffer (``Device::F`` / ``Device::U``); freed with the object."""

    def __init__(self, engine: "Engine", handle, dtype: int, owner=None):
        self.engine = engine
        self.h = handle
        self.dtype = dtype
        self._owner = owner  # keeps wrapped memory alive

    def __len__(self) -> int:
        return load().eb_buf_len(self.h)

    @property
    def ptr(self) -> int:
        return load().eb_buf_ptr(self.h) or 0

    def read(self, lo: int = 0, hi: Optional[int] = None) -> np.ndarray:
        """``Device::read_f32/u32``: waits for queued work."""
        hi = len(self) if hi is None else hi
        out = np.empty(max(hi - lo, 0), np.float32 if self.dtype == F32 else np.uint32)
        _check(load().eb_buf_read(self.engine.h, self.h, lo, hi, _ptr(out)))
        return out

    def write(self, offset: int, values) -> None:
        """``Device::write_f32/u32``."""
        v = _f32(values) if self.dtype == F32 else _u32(values)
        _check(load().eb_buf_write(self.engine.h, self.h, offset, _ptr(v), v.size))

    def free(self) -> None:
        if self.h and self.engine.h:
            load().eb_buf_free(self.engine.h, self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class Config:
    """The training inputs of ``model::Config`` (crates/emeans-core/src/model.rs:23-67)."""
    d: int
    k: int
    nepochs: float = 5.0
    batch_size: Optional[int] = None
    alpha0: Optional[float] = None
    batch_law: str = "auto"
    seed: int = 1234
    spherical: bool = False
    unused_threshold: Optional[float] = None
    assignment_chunk_size: Optional[int] = None
    capture_assignments: bool = True
    verbose: bool = False


@dataclass
class Trained:
    """``core::train::Outcome`` (core/train.rs:51-58) with the epoch statistics."""
    centroids: np.ndarray
    positions: np.ndarray
    usage: np.ndarray
    labels: Optional[np.ndarray]
    obj: list = field(default_factory=list)
    imbalance: list = field(default_factory=list)
    nsplit: list = field(default_factory=list)
    epoch_time: list = field(default_factory=list)
    n_splits: int = 0
    batch_size: int = 0
    alpha0: float = 0.0
    total_steps: int = 0


_LAWS = {"auto": 0, "throughput": 1, "quality": 2}


class Engine:
    """One engine (stream, scratch, bound data) on one CUDA device."""

    def __init__(self, device: int = 0):
        lib = load()
        h = C.c_void_p()
        _check(lib.eb_engine_create(device, C.byref(h)))
        self.h = h.value
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            load().eb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- engine
    def name(self) -> str:
        buf = C.create_string_buffer(64)
        _check(load().eb_engine_name(self.h, buf, 64))
        return buf.value.decode()

    def sync(self):
        _check(load().eb_sync(self.h))

    def flush(self):
        _check(load().eb_flush(self.h))

    def set_screen_mode(self, mode: int):
        """Top-1 path: 0 exact SIMT only, 1 auto (default), 2 tensor-core screen always.
        Results are identical in every mode."""
        _check(load().eb_set_screen_mode(self.h, mode))

    def stream(self) -> int:
        """The engine's cudaStream_t, for torch.cuda.ExternalStream and events."""
        s = C.c_void_p()
        _check(load().eb_engine_stream(self.h, C.byref(s)))
        return s.value or 0

    def device_allocations(self) -> int:
        """Device allocations the engine has made since creation."""
        c = C.c_uint64()
        _check(load().eb_device_allocations(self.h, C.byref(c)))
        return c.value

    def stats(self) -> dict:
        s = Stats()
        _check(load().eb_get_stats(self.h, C.byref(s)))
        return {f: getattr(s, f) for f, _ in Stats._fields_}

    # ---- buffers (Device::bind/upload/zeros)
    def _new(self, fn, *args, dtype=F32, owner=None) -> Buffer:
        h = C.c_void_p()
        _check(fn(self.h, *args, C.byref(h)))
        return Buffer(self, h.value, dtype, owner)

    def zeros_f32(self, n: int) -> Buffer:
        return self._new(load().eb_buf_alloc, F32, n, dtype=F32)

    def zeros_u32(self, n: int) -> Buffer:
        return self._new(load().eb_buf_alloc, U32, n, dtype=U32)

    def upload_f32(self, v) -> Buffer:
        v = _f32(v).ravel()
        return self._new(load().eb_buf_upload, F32, _ptr(v), v.size, dtype=F32)

    def upload_u32(self, v) -> Buffer:
        v = _u32(v).ravel()
        return self._new(load().eb_buf_upload, U32, _ptr(v), v.size, dtype=U32)

    def bind(self, x, d: int) -> Buffer:
        x = _f32(x).ravel()
        return self._new(load().eb_bind, _ptr(x), x.size // d, d, dtype=F32)

    def wrap(self, tensor) -> Buffer:
        """A non-owning view of a torch CUDA tensor (float32 or int32/uint32)."""
        import torch

        assert tensor.is_cuda and tensor.is_contiguous()
        dtype = F32 if tensor.dtype == torch.float32 else U32
        assert tensor.dtype in (torch.float32, torch.int32, torch.uint32)
        return self._new(load().eb_buf_wrap, dtype, tensor.data_ptr(), tensor.numel(), dtype=dtype,
                         owner=tensor)

    # ---- layer-1 ops (trait Device)
    def top1(self, x: Buffer, d: int, ids: Optional[Buffer], rows: range, centroids: Buffer,
             cnorm: Optional[Buffer], k: int, metric: int, labels: Buffer, scores: Buffer):
        _check(load().eb_top1(self.h, x.h, d, ids.h if ids else None, rows.start, rows.stop,
                              centroids.h, cnorm.h if cnorm else None, k, metric, labels.h,
                              scores.h))

    def topk(self, queries, data, d: int, kk: int, exclude_self: bool = False):
        q, x = _f32(queries).ravel(), _f32(data).ravel()
        m, n = q.size // d, x.size // d
        ids = np.empty(m * kk, np.uint32)
        sims = np.empty(m * kk, np.float32)
        _check(load().eb_topk(self.h, _ptr(q), m, _ptr(x), n, d, kk, int(exclude_self),
                              _ptr(ids), _ptr(sims)))
        return ids, sims

    def internal_scores(self, x, d: int, labels, k: int) -> dict:
        """``metrics::internal_scores`` (crates/emeans-cluster/src/metrics.rs:115-274)
        on the device: silhouette, Calinski-Harabasz, Davies-Bouldin, objective,
        k_eff and the cluster sizes of ``labels`` (values < k) on unit rows x."""
        xa, la = _f32(x).ravel(), _u32(np.asarray(labels, dtype=np.uint32).ravel())
        n = la.size
        if xa.size != n * d:
            raise ValueError("x must be n x d with one label per row")
        out = _Internal()
        sizes = np.zeros(k, np.uint64)
        _check(load().eb_internal_scores(self.h, _ptr(xa) if xa.size else None, n, d,
                                         _ptr(la) if n else None, k, C.byref(out),
                                         _ptr(sizes) if k else None))
        return {"k_eff": int(out.k_eff), "silhouette": out.silhouette,
                "calinski_harabasz": out.calinski_harabasz,
                "davies_bouldin": out.davies_bouldin, "objective": out.objective,
                "sizes": sizes}

    def dedup(self, x, d: int, created=None, burst=None, priority=None,
              cfg: Optional[DedupConfig] = None) -> "DedupResult":
        """``dedup::dedup`` (crates/emeans-cluster/src/dedup.rs:160-183): the
        exact kNN self-join on the engine, then the grouping stages."""
        cfg = cfg or DedupConfig()
        xa = _f32(x).ravel()
        n = xa.size // d
        t, b, p = _dedup_side(n, created, burst, priority)
        return _dedup_call(lambda c, o: load().eb_dedup(
            self.h, _ptr(xa), n, d, _ptr(t), _ptr(b), _ptr(p), c, o), n, cfg)

    def topk_group(self, queries, shard, shard_offset: int, n_total: int, d: int, kk: int,
                   exclude_self: bool = False):
        """eb_topk_group: top-kk over a database sharded across the engine's
        group (this rank holds rows shard_offset .. + len(shard)); collective."""
        q, x = _f32(queries).ravel(), _f32(shard).ravel()
        m, n = q.size // d, x.size // d
        ids = np.empty(m * kk, np.uint32)
        sims = np.empty(m * kk, np.float32)
        _check(load().eb_topk_group(self.h, _ptr(q), m, _ptr(x) if n else None, n, shard_offset,
                                    n_total, d, kk, int(exclude_self), _ptr(ids), _ptr(sims)))
        return ids, sims

    def scatter_add(self, x: Buffer, d: int, ids: Optional[Buffer], rows: range, labels: Buffer,
                    k: int, sums: Buffer, counts: Buffer, acc: Optional[Buffer] = None):
        _check(load().eb_scatter_add(self.h, x.h, d, ids.h if ids else None, rows.start,
                                     rows.stop, labels.h, k, sums.h, counts.h,
                                     acc.h if acc else None))

    def row_norms(self, m: Buffer, rows: int, d: int, out: Buffer):
        _check(load().eb_row_norms(self.h, m.h, rows, d, out.h))

    def normalize_rows(self, src: Buffer, rows: int, d: int, dst: Buffer):
        _check(load().eb_normalize_rows(self.h, src.h, rows, d, dst.h))

    def split(self, positions: Buffer, usage: Buffer, plan: Sequence, d: int):
        p = _u32(np.asarray(plan, dtype=np.uint32).reshape(-1))
        _check(load().eb_split(self.h, positions.h, usage.h, _ptr(p), p.size // 2, d))

    def ema_update(self, positions: Buffer, usage: Buffer, sums: Buffer, counts: Buffer, k: int,
                   d: int, alpha: float):
        """``Device::ema_update`` with ``EmaStep::new(alpha)`` (core/mod.rs:189-197)."""
        a32 = np.float32(alpha)
        decay = np.float32(1.0 - alpha)
        _check(load().eb_ema_update(self.h, positions.h, usage.h, sums.h, counts.h, k, d,
                                    float(a32), float(decay), int(alpha == 1.0)))

    # ---- Assigner::assign and the device loop
    def assign(self, rows, d: int, centroids, metric: int, ids=None):
        x = _f32(rows).ravel()
        c = _f32(centroids).ravel()
        n, k = x.size // d, c.size // d
        idv = None if ids is None else _u32(ids).ravel()
        m = n if idv is None else idv.size
        labels = np.empty(m, np.uint32)
        scores = np.empty(m, np.float32)
        _check(load().eb_assign(self.h, _ptr(x), n, d, _ptr(idv), m, _ptr(c), k, metric,
                                _ptr(labels), _ptr(scores)))
        return labels, scores

    def assign_ptr(self, x_ptr: int, n: int, d: int, c_ptr: int, k: int, metric: int,
                   labels_ptr: int, scores_ptr: int):
        """``eb_assign`` on caller-owned host memory (pinned buffers for the e2e bench)."""
        _check(load().eb_assign(self.h, x_ptr, n, d, None, n, c_ptr, k, metric, labels_ptr,
                                scores_ptr))

    def bind_data(self, data, d: int):
        x = _f32(data).ravel()
        self._bound = x  # the host copy that indexed assign calls compare against
        _check(load().eb_bind_data(self.h, _ptr(x), x.size // d, d))
        return x

    def unbind_data(self):
        _check(load().eb_unbind_data(self.h))
        self._bound = None

    def set_kernel_timing(self, on: bool):
        """Bracket every top-1 screen launch with CUDA events (measurement)."""
        _check(load().eb_set_kernel_timing(self.h, int(bool(on))))

    def screen_timing(self):
        """(summed device ms, launches, rows) of the screen launches since the
        last call; waits for queued work."""
        ms, n, r = C.c_double(), C.c_uint64(), C.c_uint64()
        _check(load().eb_screen_timing(self.h, C.byref(ms), C.byref(n), C.byref(r)))
        return ms.value, n.value, r.value

    def join(self, rank: int, world: int, group_id: bytes):
        """Join a multi-GPU group (eb_engine_join); collective over the ranks."""
        if len(group_id) != GROUP_ID_BYTES:
            raise ValueError(f"group id must be {GROUP_ID_BYTES} bytes")
        _check(load().eb_engine_join(self.h, rank, world, group_id))

    def join_torch_group(self):
        """Join with every rank of the default torch.distributed group: rank 0
        draws the id and broadcasts it (as bytes) over that group."""
        import torch.distributed as dist
        rank, world = dist.get_rank(), dist.get_world_size()
        box = [group_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        self.join(rank, world, box[0])

    def set_group_shard(self, mode: int):
        """eb_set_group_shard: 0 auto (split a training batch's top-1 across
        the group only when that shortens it), 1 always, 2 never (all three
        equal one engine bit for bit); 3 splits the top-1 and the scatter-add
        and adds the ranks' partial sums in rank order (one all-gather per
        step; equal to one engine to rounding). Same on every rank."""
        _check(load().eb_set_group_shard(self.h, int(mode)))

    def group_allgather(self, buf: "Buffer", words_per_rank: int):
        """eb_group_allgather: in-place all-gather of buf's rank shares
        (words_per_rank 32-bit words each); collective over the group."""
        _check(load().eb_group_allgather(self.h, buf.h, int(words_per_rank)))

    def group_exchange(self, words: int) -> "Buffer":
        """eb_group_exchange: a buffer of ``words`` 32-bit words in the group's
        exchange region (collective), whose all-gather runs over NVLink peer
        memory; a plain buffer when alone. The region is the engine's: keep the
        view only while the group lasts."""
        return self._new(load().eb_group_exchange, int(words), dtype=U32)

    def group_exchange_info(self):
        """(mapped, why): whether the exchange region is mapped over peer memory,
        and the reason the last set-up mapped none."""
        m = C.c_int()
        why = C.create_string_buffer(512)
        _check(load().eb_group_exchange_info(self.h, C.byref(m), why, 512))
        return bool(m.value), why.value.decode()

    def view(self, buf: "Buffer", offset: int, length: int, dtype: int) -> "Buffer":
        """A non-owning view of buf's elements offset .. offset + length
        (4-byte elements; the view's start must be 16-byte aligned). A range
        past buf's end is refused (INVALID_ARGUMENT), as the C calls refuse
        one."""
        offset, length = int(offset), int(length)
        if offset < 0 or length < 0 or offset + length > len(buf):
            raise EngineError(INVALID_ARGUMENT,
                              f"view {offset} .. {offset + length} is outside the buffer's "
                              f"{len(buf)} elements")
        return self._new(load().eb_buf_wrap, dtype, buf.ptr + 4 * offset, length,
                         dtype=dtype, owner=buf)

    def group(self):
        r, w = C.c_int(), C.c_int()
        _check(load().eb_engine_group(self.h, C.byref(r), C.byref(w)))
        return r.value, w.value

    def train(self, x, cfg: Config, init=None, state=None) -> Trained:
        """``Engine::run_train``: the device loop (core/train.rs:60-303)."""
        x = _f32(x).ravel()
        d, k = cfg.d, cfg.k
        n = x.size // d
        cent = np.empty(k * d, np.float32)
        pos = np.empty(k * d, np.float32)
        usage = np.empty(k, np.float32)
        labels = np.empty(n, np.int32) if cfg.capture_assignments else None
        init_a = None if init is None else _f32(init).ravel()
        sp = su = None
        if state is not None:
            sp, su = _f32(state[0]).ravel(), _f32(state[1]).ravel()
        job = TrainJob(x=_ptr(x), n=n, d=d, k=k, nepochs=float(cfg.nepochs),
                       batch_law=_LAWS[cfg.batch_law], spherical=int(cfg.spherical),
                       batch_size=cfg.batch_size or 0,
                       alpha0=math.nan if cfg.alpha0 is None else float(cfg.alpha0),
                       unused_threshold=math.nan if cfg.unused_threshold is None
                       else float(cfg.unused_threshold),
                       seed=cfg.seed, capture=int(cfg.capture_assignments),
                       chunk=cfg.assignment_chunk_size or 0, init=_ptr(init_a),
                       state_positions=_ptr(sp), state_usage=_ptr(su), verbose=int(cfg.verbose))
        out = TrainOut(centroids=_ptr(cent), positions=_ptr(pos), usage=_ptr(usage),
                       labels=_ptr(labels))
        _check(load().eb_train(self.h, C.byref(job), C.byref(out)))
        ne = out.n_epochs
        return Trained(centroids=cent.reshape(k, d), positions=pos.reshape(k, d), usage=usage,
                       labels=labels, obj=list(out.obj[:ne]), imbalance=list(out.imbalance[:ne]),
                       nsplit=list(out.nsplit[:ne]), epoch_time=list(out.epoch_time[:ne]),
                       n_splits=out.n_splits, batch_size=out.batch_size, alpha0=out.alpha0,
                       total_steps=out.total_steps)


    def fit(self, x, d: int, k: int, nepochs: float, seed: int, init_rows=None):
        """``auto::fit`` (crates/emeans-cluster/src/auto.rs:350-375) on the
        engine: one spherical model (``Config::new(d, k)`` with spherical,
        nepochs and seed set, assignments not captured) trained on x, from the
        rows ``init_rows[:k]`` when given (``train_from``), and x assigned to
        it by inner product (``Emeans::assign``). With x bound
        (``bind_data``), the training and the assignment both read the bound
        rows in place: a sweep of fits uploads the data once, as the
        reference's ``SharedAssigner`` shares one binding across its fits.
        Returns (Trained, labels, scores)."""
        x = _f32(x).ravel()
        cfg = Config(d=d, k=k, nepochs=float(nepochs), seed=int(seed), spherical=True,
                     capture_assignments=False)
        init = None
        if init_rows is not None:
            r = np.asarray(init_rows, np.int64).ravel()
            if r.size < k:
                raise ValueError("need k init rows")
            init = x.reshape(-1, d)[r[:k]]
        tr = self.train(x, cfg, init=init)
        labels, scores = self.assign(x, d, tr.centroids, IP)
        return tr, labels, scores

    def sweep(self, x, d: int, ks, nepochs: float, seed: int, salt: int = 0, restarts: int = 1,
              init_rows=None):
        """``auto::sweep`` (crates/emeans-cluster/src/auto.rs:455-505) on the
        engine: for every k of ks, ``restarts`` fits (``fit``, seeds from
        ``seed_for``), the one with the lowest mean objective kept (the first
        on ties; ``Assignment::mean_objective``, model.rs:127-141: the
        sequential f64 mean of 2 - 2 cos), and its labels scored by
        ``internal_scores``. ``init_rows``: one row-id list per restart (the
        k-means++ picks, whose first k rows seed the fit with k clusters) or
        None for the seeded random rows. Bind x first (``bind_data``) to keep
        the rows on the device across the fits. Returns a list of
        (k, internal scores, Trained, labels, scores, mean objective)."""
        out = []
        for k in ks:
            best = None
            for r in range(max(int(restarts), 1)):
                rows = None if init_rows is None else init_rows[r]
                tr, lab, sco = self.fit(x, d, k, nepochs, seed_for(seed, salt, k, r), rows)
                obj = mean_objective(sco, spherical=True)
                if best is None or obj < best[0]:
                    best = (obj, tr, lab, sco)
            obj, tr, lab, sco = best
            out.append((k, self.internal_scores(x, d, lab, k), tr, lab, sco, obj))
        return out


def mean_objective(scores, spherical: bool) -> float:
    """``Assignment::mean_objective`` (crates/emeans-core/src/model.rs:127-141):
    the f64 mean, summed in row order, of 2 - 2 cos (spherical) or of the
    squared distances."""
    v = np.asarray(scores, np.float32).astype(np.float64)
    if spherical:
        v = 2.0 - 2.0 * v
    return float(np.cumsum(v)[-1]) / max(v.size, 1) if v.size else 0.0


def seed_for(seed: int, salt: int, k: int, restart: int) -> int:
    """A sweep fit's seed (crates/emeans-cluster/src/auto.rs:343-348): u32
    wrapping arithmetic on the configured seed, a salt, k and the restart."""
    m = 0xFFFFFFFF
    return (seed + (salt * 7919 & m) + (k * 131 & m) + (restart * 1_000_003 & m)) & m


GROUP_ID_BYTES = 128


def group_unique_id() -> bytes:
    """A fresh multi-GPU group id (eb_group_unique_id), made on rank 0."""
    buf = C.create_string_buffer(GROUP_ID_BYTES)
    _check(load().eb_group_unique_id(buf))
    return buf.raw


def merge_topk(lists, kk: int):
    """The group top-k merge rule (k_topk_merge) on the host: per query, the
    best kk of the ranks' (ids, sims) lists by (larger score, then lower id),
    missing entries (id 0xFFFFFFFF) dropped and padded back at the end."""
    m = lists[0][0].size // kk
    ids = np.full(m * kk, 0xFFFFFFFF, np.uint32)
    sims = np.full(m * kk, -np.inf, np.float32)
    for qi in range(m):
        cand = [(float(s[qi * kk + t]), int(i[qi * kk + t])) for i, s in lists for t in range(kk)
                if i[qi * kk + t] != 0xFFFFFFFF]
        cand.sort(key=lambda c: (-c[0], c[1]))
        for t, (v, j) in enumerate(cand[:kk]):
            ids[qi * kk + t] = j
            sims[qi * kk + t] = v
    return ids, sims


def shard_bounds(b: int, end: int, rank: int, world: int):
    """The positions [lo, hi) of batch [b, end) that `rank` scores in a group
    of `world` engines (the split eb_train uses: equal slices of ceil(B/world),
    the last ones shorter or empty)."""
    sh = (end - b + world - 1) // world
    lo = min(b + rank * sh, end)
    hi = min(lo + sh, end) if world > 1 else end
    return lo, hi


@dataclass
class DedupConfig:
    """``dedup::DedupConfig`` (crates/emeans-cluster/src/dedup.rs:39-62)."""
    k: int = 10
    sim_threshold: float = 0.95
    rep_threshold: Optional[float] = None
    max_gap_secs: Optional[float] = None


@dataclass
class DedupResult:
    """``dedup::DedupResult`` (dedup.rs:77-130)."""
    group_of: np.ndarray
    representatives: np.ndarray
    anchors: np.ndarray
    sizes: np.ndarray
    nn_sim: np.ndarray
    linked_pairs: int
    split_components: int

    def n_groups(self) -> int:
        return int(self.representatives.size)

    def expand(self, rep_labels):
        """Every row gets its group representative's label (dedup.rs:113-120)."""
        rep_labels = np.asarray(rep_labels)
        assert rep_labels.shape[0] == self.n_groups()
        return rep_labels[self.group_of]

    def gather(self, x, d: int):
        """The representative rows, in group order (dedup.rs:123-129)."""
        return np.asarray(x, np.float32).reshape(-1, d)[self.representatives]


def _dedup_side(n, created, burst, priority):
    t = None if created is None else np.ascontiguousarray(created, np.float64)
    b = None
    if burst is not None:
        b = np.array([NONE_ID if v is None else int(v) for v in burst], np.uint32)
        if np.any(np.array([v is not None and int(v) == NONE_ID for v in burst])):
            raise ValueError("burst id 0xFFFFFFFF is reserved for no burst")
    p = None if priority is None else np.ascontiguousarray(priority, np.float32)
    for a in (t, b, p):
        if a is not None and a.size != n:
            raise ValueError("one timestamp / burst id / priority per row")
    return t, b, p


def _dedup_call(fn, n, cfg: DedupConfig):
    c = _DedupConfig(k=cfg.k, sim_threshold=cfg.sim_threshold,
                     rep_threshold=math.nan if cfg.rep_threshold is None else cfg.rep_threshold,
                     max_gap_secs=math.nan if cfg.max_gap_secs is None else cfg.max_gap_secs)
    arrs = [np.zeros(max(n, 1), np.uint32) for _ in range(4)] + [np.zeros(max(n, 1), np.float32)]
    out = _DedupOut(*[a.ctypes.data for a in arrs])
    _check(fn(C.byref(c), C.byref(out)))
    g = int(out.n_groups)
    return DedupResult(group_of=arrs[0][:n].copy(), representatives=arrs[1][:g].copy(),
                       anchors=arrs[2][:g].copy(), sizes=arrs[3][:g].copy(),
                       nn_sim=arrs[4][:n].copy(), linked_pairs=int(out.linked_pairs),
                       split_components=int(out.split_components))


def dedup_with_neighbors(x, d: int, ids, sims, kk: int, created=None, burst=None, priority=None,
                         cfg: Optional[DedupConfig] = None) -> DedupResult:
    """``dedup::dedup_with_neighbors`` (dedup.rs:186-358) on the host (C++):
    groups from the self-join neighbours ids / sims (n x kk)."""
    cfg = cfg or DedupConfig()
    xa = _f32(x).ravel()
    n = xa.size // d
    ia, sa = _u32(ids).ravel(), _f32(sims).ravel()
    if ia.size != n * kk or sa.size != n * kk:
        raise ValueError("ids and sims must be n x kk")
    t, b, p = _dedup_side(n, created, burst, priority)
    return _dedup_call(lambda c, o: load().eb_dedup_with_neighbors(
        _ptr(xa), n, d, _ptr(ia), _ptr(sa), kk, _ptr(t), _ptr(b), _ptr(p), c, o), n, cfg)


def reduce_layout(batch: int, world: int, k: int, d: int):
    """The per-rank share of eb_train's exchange buffer in group mode 3 (the
    split top-1 and scatter-add): (s, s4, k4, share) with s = ceil(batch /
    world) positions per rank; labels at [0, s4), scores at [s4, 2 s4),
    partial counts at [2 s4, 2 s4 + k), partial sums (k x d) at
    [2 s4 + k4, share), all in 32-bit words (s4, k4: s and k rounded up to 4)."""
    s = (batch + world - 1) // world
    s4, k4 = (s + 3) // 4 * 4, (k + 3) // 4 * 4
    return s, s4, k4, 2 * s4 + k4 + k * d


class B200Assigner:
    """``trait Assigner`` (crates/emeans-core/src/assign.rs:71-117) on the engine."""

    def __init__(self, device: int = 0):
        self.engine = Engine(device)
        self._bound = None

    def name(self) -> str:
        return self.engine.name()

    def bind_data(self, data, d: int):
        self._bound = self.engine.bind_data(data, d)

    def unbind_data(self):
        self.engine.unbind_data()
        self._bound = None

    def with_engine(self, f):
        return f(self.engine)

    def assign(self, rows, d: int, centroids, metric: int, ids=None):
        if ids is not None and self._bound is not None and rows is not None and \
                np.asarray(rows).size == self._bound.size:
            rows = self._bound
        return self.engine.assign(rows, d, centroids, metric, ids=ids)


def _search(queries, data, d, k, exclude_self, engine=None):
    if k < 1 or k > GPU_KMAX:
        raise ValueError(f"k must be 1..={GPU_KMAX} on the B200 engine")
    eng = engine or Engine(0)
    ids, sims = eng.topk(queries, data, d, k, exclude_self)
    m = ids.size // k
    return ids.reshape(m, k), sims.reshape(m, k)


def dedup(x, d: int, created=None, burst=None, priority=None,
          cfg: Optional[DedupConfig] = None, engine: Optional[Engine] = None) -> DedupResult:
    """Near-duplicate groups of the unit rows x (dedup.rs:160-183) on the B200."""
    return (engine or Engine(0)).dedup(x, d, created, burst, priority, cfg)


def knn_self(data, d: int, k: int, engine: Optional[Engine] = None):
    """Neighbours of every row among the other rows (knn.rs:17-19)."""
    return _search(data, data, d, k, True, engine)


def knn(queries, data, d: int, k: int, engine: Optional[Engine] = None):
    """Neighbours of every query row among the data rows (knn.rs:21-29)."""
    return _search(queries, data, d, k, False, engine)
