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


PLAN_DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include "host.h"
// argv: seed tau rounds k; stdin: rounds x k float32 usage vectors. Plans each
// round in turn with one generator, drawing the uniforms ahead on odd rounds
// (as the training loop does) and inside plan_revival on even ones.
int main(int argc, char** argv) {
  const uint32_t seed = (uint32_t)strtoul(argv[1], nullptr, 10);
  const double tau = strtod(argv[2], nullptr);
  const size_t rounds = (size_t)strtoull(argv[3], nullptr, 10);
  const size_t k = (size_t)strtoull(argv[4], nullptr, 10);
  eb::host::Mt19937 rng(seed);
  std::vector<float> u(k);
  for (size_t r = 0; r < rounds; r++) {
    if (fread(u.data(), 4, k, stdin) != k) return 2;
    eb::host::RevivalDraws pre = eb::host::revival_draws(rng, k);
    std::vector<uint32_t> plan = eb::host::plan_revival(u, tau, rng, (r & 1) ? &pre : nullptr);
    printf("%zu", plan.size() / 2);
    for (uint32_t v : plan) printf(" %u", v);
    printf("\n");
  }
  return 0;
}
"""


@pytest.fixture(scope="module")
def plan_driver(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not found")
    d = tmp_path_factory.mktemp("host_plan")
    src, exe = d / "plan.cpp", d / "plan"
    src.write_text(PLAN_DRIVER)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    return str(exe)


@pytest.mark.parametrize("k", [1, 2, 7, 64, 1024, 5000])
def test_revival_plan_matches_oracle(plan_driver, k):
    """The engine's host revival plan (csrc/host.h) against the oracle's
    restatement of core/mod.rs:339-370 over a run of revivals sharing one
    generator: the same pairs in the same order, and the same draws."""
    rs = np.random.default_rng(k)
    rounds, tau, seed = 8, 0.5, 4321
    usage = []
    for r in range(rounds):
        u = rs.exponential(1.0, k).astype(np.float32) * np.float32(10.0 ** rs.uniform(-6, 2))
        dead = rs.random(k) < [0.0, 0.05, 0.4, 0.9, 0.3, 0.6, 0.0, 0.2][r]
        u[dead] = np.float32(0.0) if r % 2 else u[dead] * np.float32(1e-6)
        if r == 5:
            u[: k // 2] = u[0]  # ties in usage: equal log terms
        usage.append(u)
    out = subprocess.run([plan_driver, str(seed), repr(tau), str(rounds), str(k)],
                         input=np.concatenate(usage).tobytes(), check=True,
                         capture_output=True).stdout.decode().splitlines()
    ref = oracle.Rng(seed)
    for r in range(rounds):
        want = ref.plan_revival(usage[r], tau)
        got = [int(v) for v in out[r].split()]
        assert got[0] == len(want), (r, got[0], len(want))
        pairs = list(zip(got[1::2], got[2::2]))
        assert pairs == want, r


def test_sweep_seed_wraps_like_u32():
    """auto.rs:343-348: seed + salt 7919 + k 131 + restart 1,000,003, each
    product and sum wrapping at 2^32."""
    import emeans_b200 as eb

    m = 2 ** 32
    for seed, salt, k, restart in [(7, 3, 64, 2), (2 ** 32 - 1, 1, 1, 1), (123, 2 ** 31, 2 ** 20, 5000),
                                   (0, 0, 0, 0)]:
        want = seed
        for term in (salt * 7919 % m, k * 131 % m, restart * 1_000_003 % m):
            want = (want + term) % m
        assert eb.seed_for(seed, salt, k, restart) == want
