"""The hot kernels keep their working sets in registers.

ptxas reports, per kernel, the bytes of local memory (stack frame) and spills.
The tensor-core screen holds a drained tile (128 accumulator values per
thread) in registers between TMEM and the scoring; if the compiler ever
indexes that array at run time, it moves to local memory and the screen slows
down by half without any change in its results. This test compiles the
screen's translation unit for sm_100a (no GPU needed) and checks that every
screen instantiation and the exact pairs kernel use no local memory; the
metrics kernels likewise.
"""

import os
import re
import subprocess

import pytest

from emeans_b200 import build as ebuild

HERE = os.path.dirname(os.path.abspath(__file__))


def _ptxas_report(src: str) -> str:
    cmd = [ebuild.nvcc(), "-x", "cu", *ebuild.ARCH, *ebuild.COMMON, "-Xptxas", "-v", "-c",
           os.path.join(ebuild.CSRC, src), "-o", os.devnull]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]
    return res.stderr


def _local_memory(src: str) -> dict:
    """Per kernel of src: (stack frame, spill stores, spill loads) bytes."""
    rep = _ptxas_report(src)
    found = {}
    cur = None
    for line in rep.splitlines():
        m = re.search(r"Function properties for (\S+)", line)
        if m:
            cur = m.group(1)
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and cur:
            found[cur] = tuple(int(v) for v in m.groups())
            cur = None
    return found


@pytest.mark.timeout(600)
def test_metrics_kernels_use_no_local_memory():
    """The metrics product keeps its 8 x 8 accumulator tile and the eight rows'
    f64 state in registers."""
    try:
        ebuild.nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    found = _local_memory("metrics.cu")
    names = ["k_silhouette", "k_db", "k_sum64", "k_cluster_prep", "k_grand"]
    for want in names:
        hits = {k: v for k, v in found.items() if want in k}
        assert hits, (want, sorted(found))
        for name, (stack, st, ld) in hits.items():
            assert stack == 0 and st == 0 and ld == 0, (name, stack, st, ld)


@pytest.mark.timeout(600)
def test_screen_and_pairs_use_no_local_memory():
    try:
        ebuild.nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    found = _local_memory("top1_tc.cu")
    screens = {k: v for k, v in found.items() if "k_screen" in k}
    pairs = {k: v for k, v in found.items() if "k_pairsILb" in k}
    # top-1 L2, top-1 IP, top-k, and the internal scores' product mode
    assert len(screens) == 4, sorted(found)
    assert pairs, sorted(found)
    for name, (stack, st, ld) in {**screens, **pairs}.items():
        assert stack == 0 and st == 0 and ld == 0, (name, stack, st, ld)
