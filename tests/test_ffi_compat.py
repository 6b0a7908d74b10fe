"""libemeans.so, the reference's C FFI for assign (include/emeans.h) over the
B200 engine: the reference's symbols, status codes and error rules
(crates/emeans-ffi/src/lib.rs:124-219, 387-408, 784-825), and on a GPU its
results against the oracle.

The CPU tests call only paths that fail before any device work (or, with no
GPU, the engine's own no-device error)."""
import ctypes as C
import json
import os
import pathlib
import re

import numpy as np
import pytest

import emeans_b200
from tests.conftest import has_gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "emeans.h"
OK, INVALID, ERROR = 0, 1, 2
F32, U32 = 0, 1


class Array(C.Structure):
    _fields_ = [("data", C.c_void_p), ("len", C.c_size_t), ("dtype", C.c_int32)]


@pytest.fixture(scope="module")
def ffi():
    emeans_b200.load()  # builds nothing; fails loudly if the engine library is missing
    path = os.path.join(os.path.dirname(emeans_b200.__file__), "libemeans.so")
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: run emeans_b200.build.build()")
    lib = C.CDLL(path)
    lib.emeans_abi_version.restype = C.c_uint32
    lib.emeans_version.restype = C.c_char_p
    lib.emeans_last_error.restype = C.c_char_p
    lib.emeans_result_json.restype = C.c_char_p
    lib.emeans_result_json.argtypes = [C.c_void_p]
    lib.emeans_result_free.argtypes = [C.c_void_p]
    lib.emeans_string_free.argtypes = [C.c_void_p]
    lib.emeans_backends.argtypes = [C.POINTER(C.c_void_p)]
    lib.emeans_assign.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                  C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p)]
    lib.emeans_result_array.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(Array)]
    lib.emeans_default_config.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    lib.emeans_train.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_char_p,
                                 C.POINTER(C.c_void_p)]
    lib.emeans_model_train.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                       C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
    lib.emeans_model_assign.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]
    lib.emeans_model_objective.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t,
                                           C.POINTER(C.c_double)]
    lib.emeans_model_centroids.argtypes = [C.c_void_p, C.POINTER(Array)]
    lib.emeans_model_info.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    lib.emeans_model_free.argtypes = [C.c_void_p]
    return lib


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(emeans_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol(ffi):
    names = declared()
    assert "emeans_assign" in names and "emeans_result_array" in names
    assert [n for n in names if not hasattr(ffi, n)] == []


def test_version_and_abi(ffi):
    assert ffi.emeans_abi_version() == 1
    assert re.fullmatch(rb"\d+\.\d+\.\d+", ffi.emeans_version())


def assign(ffi, x, c, d, metric=b"l2", backend=None, n=None, k=None, xp=None, cp=None):
    out = C.c_void_p()
    n = len(x) // d if n is None else n
    k = len(c) // d if k is None else k
    xp = x.ctypes.data if xp is None else xp
    cp = c.ctypes.data if cp is None else cp
    rc = ffi.emeans_assign(xp, n, d, cp, k, metric, backend, C.byref(out))
    return rc, out


def test_argument_errors_are_invalid_argument(ffi):
    x = np.zeros(64, np.float32)
    c = np.zeros(16, np.float32)
    assert ffi.emeans_assign(x.ctypes.data, 4, 16, c.ctypes.data, 1, b"l2", None, None) == INVALID
    assert b"out_result is NULL" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, xp=0)
    assert rc == INVALID and b"data is NULL" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, cp=0)
    assert rc == INVALID and b"centroids is NULL" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, xp=x.ctypes.data + 2)
    assert rc == INVALID and b"not aligned" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, n=2**62)
    assert rc == INVALID and b"overflows" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, metric=None)
    assert rc == INVALID and b"metric is NULL" in ffi.emeans_last_error()


def test_shape_metric_and_backend_errors(ffi):
    x = np.zeros(64, np.float32)
    c = np.zeros(16, np.float32)
    rc, _ = assign(ffi, x, c, 0, n=4, k=1)
    assert rc == ERROR and b"d must be positive" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, k=0)
    assert rc == ERROR and b"centroids is empty" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, metric=b"manhattan")
    assert rc == ERROR and b"unknown metric" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, backend=b"cpu-gemm")
    assert rc == ERROR and b"not in this library" in ffi.emeans_last_error()
    rc, _ = assign(ffi, x, c, 16, backend=b"tpu")
    assert rc == ERROR and b"unknown backend" in ffi.emeans_last_error()


def test_null_handles(ffi):
    arr = Array()
    assert ffi.emeans_result_array(None, b"labels", C.byref(arr)) == INVALID
    assert ffi.emeans_result_json(None) is None
    ffi.emeans_result_free(None)
    ffi.emeans_string_free(None)


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_no_device_is_an_error_not_a_fallback(ffi):
    x = np.ones(64, np.float32)
    c = np.ones(16, np.float32)
    rc, out = assign(ffi, x, c, 16)
    assert rc == ERROR and b"no B200 engine" in ffi.emeans_last_error()
    assert not out.value
    s = C.c_void_p()
    assert ffi.emeans_backends(C.byref(s)) == OK
    assert ffi.emeans_last_error() is None
    assert json.loads(C.string_at(s.value)) == []
    ffi.emeans_string_free(s)


def read(ffi, r, name):
    arr = Array()
    assert ffi.emeans_result_array(r, name, C.byref(arr)) == OK
    if arr.len == 0:
        assert arr.data is None
        return np.zeros(0), arr.dtype
    ct = C.c_float if arr.dtype == F32 else C.c_uint32
    return np.ctypeslib.as_array(C.cast(arr.data, C.POINTER(ct)), (arr.len,)).copy(), arr.dtype


@pytest.mark.gpu
@pytest.mark.parametrize("metric,code", [(b"l2", 0), (b"inner_product", 1), (b"cosine", 1)])
def test_assign_matches_oracle(ffi, metric, code):
    import oracle

    rng = np.random.default_rng(11)
    n, d, k = 3000, 72, 257
    x = rng.standard_normal((n, d)).astype(np.float32)
    c = x[rng.permutation(n)[:k]] * np.float32(1.01)
    c[5] = c[4]  # a duplicate centroid: ties keep the lower id
    # "cpu" (the reference default, the fused kernel on x86_64) and
    # "cpu-fused" are served by the engine with the same bits.
    for backend in (None, b"cuda", b"cpu", b"cpu-fused"):
        rc, r = assign(ffi, x.ravel(), c.ravel(), d, metric=metric, backend=backend)
        assert rc == OK, ffi.emeans_last_error()
        assert ffi.emeans_last_error() is None
        labels, lt = read(ffi, r, b"labels")
        scores, st = read(ffi, r, b"scores")
        assert (lt, st) == (U32, F32)
        assert json.loads(ffi.emeans_result_json(r)) == {}
        arr = Array()
        assert ffi.emeans_result_array(r, b"centroids", C.byref(arr)) == ERROR
        assert b"has: labels, scores" in ffi.emeans_last_error()
        ffi.emeans_result_free(r)
        wl, ws = oracle.top1(x.ravel(), d, c.ravel(), code)
        assert np.array_equal(labels, wl)
        assert np.array_equal(scores.astype(np.float32).view(np.uint32), ws.view(np.uint32))


@pytest.mark.gpu
def test_assign_empty_and_backends(ffi):
    c = np.ones(32, np.float32)
    out = C.c_void_p()
    assert ffi.emeans_assign(None, 0, 16, c.ctypes.data, 2, b"l2", None, C.byref(out)) == OK
    labels, _ = read(ffi, out, b"labels")
    assert labels.size == 0
    ffi.emeans_result_free(out)
    s = C.c_void_p()
    assert ffi.emeans_backends(C.byref(s)) == OK
    assert json.loads(C.string_at(s.value)) == ["cuda"]
    ffi.emeans_string_free(s)


def take_string(ffi, p):
    v = C.string_at(p.value).decode()
    ffi.emeans_string_free(p)
    return v


def test_default_config(ffi):
    s = C.c_void_p()
    assert ffi.emeans_default_config(b"train", C.byref(s)) == OK
    cfg = json.loads(take_string(ffi, s))
    assert cfg["nepochs"] == 5.0 and cfg["seed"] == 1234 and cfg["batch_law"] == "auto"
    assert cfg["capture_assignments"] is True and cfg["exact_objective"] is False
    assert cfg["backend"] == "cuda" and "d" not in cfg and "k" not in cfg
    assert ffi.emeans_default_config(b"auto", C.byref(s)) == ERROR
    assert b"not in this library" in ffi.emeans_last_error()
    assert ffi.emeans_default_config(b"nope", C.byref(s)) == ERROR
    assert ffi.emeans_default_config(None, C.byref(s)) == INVALID


def train_call(ffi, x, n, d, k, cfg):
    out = C.c_void_p()
    rc = ffi.emeans_train(x.ctypes.data, n, d, k, cfg, C.byref(out))
    return rc, out


def test_train_config_errors_before_any_device_work(ffi):
    x = np.zeros(64 * 4, np.float32)
    cases = [
        (b"{nope", INVALID, b"not valid JSON"),
        (b"[1, 2]", ERROR, b"config must be an object"),
        (b'{"d": 4}', ERROR, b"pass d as an argument"),
        (b'{"epochs": 3}', ERROR, b"unknown config key \"epochs\" (known: alpha0,"),
        (b'{"exact_objective": 1}', ERROR, b"exact_objective\" must be true or false"),
        (b'{"backend": "cpu-accelerate"}', ERROR, b"not in this library"),
        (b'{"backend": "\\ud800"}', INVALID, b"not valid JSON"),
        (b'{"backend": "\\udc00x"}', INVALID, b"not valid JSON"),
        (b'{"backend": "\\ud83d\\u0041"}', INVALID, b"not valid JSON"),
        (b'{"backend": "\\ud83d\\ude00"}', ERROR, "unknown backend \"\U0001F600\"".encode()),
        (b'{"backend": 3}', ERROR, b"must be a string"),
        (b'{"seed": -1}', ERROR, b"bad train config"),
        (b'{"batch_size": 2.5}', ERROR, b"bad train config"),
        (b'{"batch_law": "fast"}', ERROR, b"bad train config"),
        (b'{"spherical": "yes"}', ERROR, b"bad train config"),
    ]
    for cfg, code, msg in cases:
        rc, out = train_call(ffi, x, 64, 4, 8, cfg)
        assert rc == code, (cfg, rc, ffi.emeans_last_error())
        assert msg in ffi.emeans_last_error(), (cfg, ffi.emeans_last_error())
        assert not out.value
    rc, _ = train_call(ffi, x, 64, 0, 8, None)
    assert rc == ERROR and b"d must be positive" in ffi.emeans_last_error()
    rc, _ = train_call(ffi, x, 64, 4, 0, None)
    assert rc == ERROR and b"k must be positive" in ffi.emeans_last_error()
    rc, _ = train_call(ffi, x, 4, 4, 8, None)
    assert rc == ERROR and b"need at least k = 8 rows, got 4" in ffi.emeans_last_error()
    assert ffi.emeans_train(x.ctypes.data, 64, 4, 8, None, None) == INVALID
    m = C.c_void_p()
    assert ffi.emeans_model_train(x.ctypes.data, 64, 4, 8, None, None, None) == INVALID
    assert ffi.emeans_model_assign(None, x.ctypes.data, 1, C.byref(m)) == INVALID
    assert b"model is NULL" in ffi.emeans_last_error()
    d_ = C.c_double()
    assert ffi.emeans_model_objective(None, x.ctypes.data, 1, C.byref(d_)) == INVALID
    ffi.emeans_model_free(None)


def blobs(seed, n, d, k):
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((k, d)).astype(np.float32) * 3
    return (means[rng.integers(0, k, n)] + rng.standard_normal((n, d))).astype(np.float32)


def unit(x):
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("spherical", [False, True])
def test_train_matches_oracle(ffi, spherical):
    import oracle

    n, d, k = 6000, 24, 40
    x = blobs(3, n, d, k)
    if spherical:
        x = unit(x)
    cfg = {"nepochs": 3.0, "seed": 77, "spherical": spherical, "exact_objective": True}
    rc, r = train_call(ffi, x, n, d, k, json.dumps(cfg).encode())
    assert rc == OK, ffi.emeans_last_error()
    cent, ct = read(ffi, r, b"centroids")
    arr = Array()
    assert ffi.emeans_result_array(r, b"labels", C.byref(arr)) == OK and arr.dtype == 2
    labels = np.ctypeslib.as_array(C.cast(arr.data, C.POINTER(C.c_int32)), (arr.len,)).copy()
    meta = json.loads(ffi.emeans_result_json(r))
    ffi.emeans_result_free(r)
    want = oracle.train(x, d, k, nepochs=3.0, seed=77, spherical=spherical)
    assert ct == F32
    assert np.array_equal(cent.astype(np.float32).view(np.uint32), want["centroids"].view(np.uint32))
    assert np.array_equal(labels, want["labels"])
    assert meta["k"] == k and meta["d"] == d and meta["backend"] == "b200"
    assert [s["obj"] for s in meta["stats"]] == want["obj"]
    assert [s["nsplit"] for s in meta["stats"]] == want["nsplit"]
    rec = oracle.recipe(n, k, d, 3.0)
    assert meta["objective"] == want["obj"][-1] / rec["epoch_rows"][-1]
    _, scores = oracle.top1(x, d, want["centroids"], oracle.IP if spherical else oracle.L2)
    s64 = scores.astype(np.float64)
    terms = 2.0 - 2.0 * s64 if spherical else s64
    assert meta["exact_objective"] == float(np.cumsum(terms)[-1] / n)


@pytest.mark.gpu
def test_model_calls_and_training_subset(ffi):
    import oracle

    n, d, k = 5000, 16, 20
    x = blobs(4, n, d, k)
    cfg = json.dumps({"nepochs": 2.0, "seed": 5, "max_points_per_centroid": 100}).encode()
    m, r = C.c_void_p(), C.c_void_p()
    assert ffi.emeans_model_train(x.ctypes.data, n, d, k, cfg, C.byref(m), C.byref(r)) == OK, \
        ffi.emeans_last_error()
    # The subset: the first 100 k of an MT19937 permutation (seed ^ 0x9E3779B9), sorted.
    keep = np.sort(oracle.permutation(5 ^ 0x9E3779B9, n)[:100 * k].astype(np.int64))
    want = oracle.train(x[keep], d, k, nepochs=2.0, seed=5)
    arr = Array()
    assert ffi.emeans_model_centroids(m, C.byref(arr)) == OK and arr.len == k * d
    cent = np.ctypeslib.as_array(C.cast(arr.data, C.POINTER(C.c_float)), (arr.len,)).copy()
    assert np.array_equal(cent.view(np.uint32), want["centroids"].view(np.uint32))
    assert ffi.emeans_result_array(r, b"labels", C.byref(arr)) == OK and arr.len == n
    labels = np.ctypeslib.as_array(C.cast(arr.data, C.POINTER(C.c_int32)), (n,)).copy()
    expect = np.full(n, -1, np.int32)
    expect[keep] = want["labels"]
    assert np.array_equal(labels, expect)
    ffi.emeans_result_free(r)
    s = C.c_void_p()
    assert ffi.emeans_model_info(m, C.byref(s)) == OK
    info = json.loads(take_string(ffi, s))
    assert info == {"d": d, "k": k, "metric": "l2", "spherical": False, "backend": "b200",
                    "epochs": len(want["obj"])}
    out = C.c_void_p()
    assert ffi.emeans_model_assign(m, x.ctypes.data, n, C.byref(out)) == OK
    got_l, _ = read(ffi, out, b"labels")
    got_s, _ = read(ffi, out, b"scores")
    ffi.emeans_result_free(out)
    wl, ws = oracle.top1(x, d, want["centroids"], oracle.L2)
    assert np.array_equal(got_l, wl)
    assert np.array_equal(got_s.astype(np.float32).view(np.uint32), ws.view(np.uint32))
    obj = C.c_double()
    assert ffi.emeans_model_objective(m, x.ctypes.data, n, C.byref(obj)) == OK
    assert obj.value == float(np.cumsum(ws.astype(np.float64))[-1] / n)
    ffi.emeans_model_free(m)
    # max_points_per_centroid * k past 2^64 - 1: the limit is above any n, so
    # every row trains (no wrap-around to a small sample).
    big = json.dumps({"nepochs": 2.0, "seed": 5, "max_points_per_centroid": 2 ** 62}).encode()
    rc, r = train_call(ffi, x, n, d, k, big)
    assert rc == OK, ffi.emeans_last_error()
    cent, _ = read(ffi, r, b"centroids")
    ffi.emeans_result_free(r)
    full = oracle.train(x, d, k, nepochs=2.0, seed=5)
    assert np.array_equal(cent.astype(np.float32).view(np.uint32), full["centroids"].view(np.uint32))


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "emeans.h"

int main(void) {
  if (emeans_abi_version() != EMEANS_ABI_VERSION) return 1;
  char* cfg = NULL;
  if (emeans_default_config("train", &cfg) != EMEANS_OK || !strstr(cfg, "\"nepochs\"")) return 2;
  emeans_string_free(cfg);
  float rows[8] = {0}, cents[4] = {0};
  EmeansResult* r = NULL;
  if (emeans_assign(rows, 2, 4, cents, 1, "hamming", NULL, &r) != EMEANS_ERROR) return 3;
  if (!emeans_last_error() || !strstr(emeans_last_error(), "unknown metric")) return 4;
  if (emeans_train(rows, 2, 4, 1, "{\"epochs\": 1}", &r) != EMEANS_ERROR) return 5;
  EmeansModel* m = NULL;
  if (emeans_model_train(rows, 2, 4, 1, "not json", &m, NULL) != EMEANS_INVALID_ARGUMENT) return 6;
  EmeansArray a;
  if (emeans_model_centroids(NULL, &a) != EMEANS_INVALID_ARGUMENT) return 7;
  emeans_result_free(NULL);
  emeans_model_free(NULL);
  printf("ok %s\n", emeans_version());
  return 0;
}
"""


def test_c_program_against_the_header_links_and_runs(tmp_path):
    """A C11 program written against include/emeans.h compiles, links against
    libemeans.so and gets the reference's status codes (no device work)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = os.path.dirname(emeans_b200.__file__)
    src, exe = tmp_path / "app.c", tmp_path / "app"
    src.write_text(C_PROGRAM)
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src),
                    "-o", str(exe), "-L", libdir, "-lemeans", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok 0.1.0")
