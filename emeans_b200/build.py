"""Build libemeans_b200.so in-tree with nvcc for sm_100a.

Every translation unit under csrc/ is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into
emeans_b200/libemeans_b200.so next to this file. Object files go to
_build/ at the repository root. Usage: ``python -m emeans_b200.build``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libemeans_b200.so")
BUILD = os.path.join(ROOT, "_build", "emeans_b200")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -ffp-contract=off keeps the host-side float order (revival plan, closing
# means, statistics) free of FMA contraction, like the reference's Rust.
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off,-O3",
          "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    deps = [src] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    deps.append(os.path.join(ROOT, "include", "emeans_b200.h"))
    return os.path.getmtime(obj) < max(os.path.getmtime(p) for p in deps)


def compile_one(src: str, verbose: bool) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    if _stale(obj, path):
        cmd = [nvcc(), *ARCH, *COMMON, "-c", path, "-o", obj]
        if src.endswith(".cu"):
            cmd[1:1] = ["-x", "cu"]
            if os.environ.get("EMEANS_B200_PTXAS_V"):
                cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", OUT, *objs, "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    build_ffi(verbose)
    return OUT


FFI_SRC = os.path.join(HERE, "ffi", "emeans_ffi.cpp")
FFI_OUT = os.path.join(HERE, "libemeans.so")


def build_ffi(verbose: bool = False) -> str:
    """libemeans.so: the reference's C FFI for assign (include/emeans.h), host
    code over libemeans_b200.so, found next to it through the run path."""
    deps = [FFI_SRC, OUT, os.path.join(ROOT, "include", "emeans.h"),
            os.path.join(ROOT, "include", "emeans_b200.h"), os.path.join(CSRC, "host.h")]
    if os.path.exists(FFI_OUT) and os.path.getmtime(FFI_OUT) >= max(os.path.getmtime(p) for p in deps):
        return FFI_OUT
    # nvcc drives the host compiler and linker as for libemeans_b200.so (the
    # same C++ runtime); the library makes no CUDA calls of its own.
    cmd = [nvcc(), *ARCH, "-O2", "-std=c++17", "-cudart", "none", "-Xcompiler", "-fPIC", "-shared",
           "-Xcompiler", "-ffp-contract=off", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
           FFI_SRC, "-o", FFI_OUT, "-L" + HERE,
           "-lemeans_b200", "-Xlinker", "-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return FFI_OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
