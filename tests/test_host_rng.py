"""The product's host-side row order (csrc/host.h: Mt19937::permutation_into,
the training loop's epoch orders and its initial centroid pick) against the
oracle's permutation and the golden MT19937 streams, on the CPU.

host.h is header-only C++, so the test compiles a small driver for it with
g++ and reads the permutations it prints.
"""
import json
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "emeans_b200", "csrc")

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include "host.h"
int main(int argc, char** argv) {
  const uint32_t seed = (uint32_t)strtoul(argv[1], nullptr, 10);
  const size_t n = (size_t)strtoull(argv[2], nullptr, 10);
  eb::host::Mt19937 g(seed);
  std::vector<uint32_t> p(n);
  g.permutation_into(p.data(), n);
  for (size_t i = 0; i < n; i++) printf("%u\n", p[i]);
  return 0;
}
"""


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not found")
    d = tmp_path_factory.mktemp("host_rng")
    src, exe = d / "perm.cpp", d / "perm"
    src.write_text(DRIVER)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    return str(exe)


def run(driver, seed, n):
    out = subprocess.run([driver, str(seed), str(n)], check=True, capture_output=True, text=True).stdout
    return np.array(out.split(), dtype=np.int64)


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 5, 8, 9, 1023, 1024, 1025, 65536, 65537, 200000])
def test_permutation_matches_oracle(driver, n):
    for seed in (0, 1234, 4294967295):
        got = run(driver, seed, n)
        want = oracle.permutation(seed, n).astype(np.int64)
        assert np.array_equal(got, want), (seed, n)
        assert sorted(got.tolist()) == list(range(n))


def test_permutation_matches_golden(driver):
    with open(os.path.join(HERE, "golden", "golden.json")) as f:
        golden = json.load(f)
    cases = [c for c in golden["mt19937"] if "random_sample" not in c]
    assert cases
    for c in cases:
        got = run(driver, c["seed"], c["n"])
        assert got[:len(c["head"])].tolist() == c["head"]
        if "tail" in c:
            assert got[len(got) - len(c["tail"]):].tolist() == c["tail"]
        m = min(c["n"], 5000)
        assert int(got[:m] @ np.arange(m)) == c["sum"]
