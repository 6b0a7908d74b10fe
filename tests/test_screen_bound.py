"""The fixed-point top-1 screen's error bound, checked on the CPU.

The screen (emeans_b200/csrc/top1_tc.cu) scales each row by s = 32638 / max|x|
(FP32), rounds to integers v = rint(fl(x s)), keeps them as int8 digits
v = 256 hi + lo, sums hi.hi and hi.lo + lo.hi exactly on the tensor cores, and
scores a = fl(hi.hi + floor((hi.lo + lo.hi) / 256)) in units of 65536; the
exact stage then decides among the centroids whose scores lie within the
window 2e of the best. That is exact only if |65536 a - x'.c'| + |chain error|
<= e for every pair, with e from screen_bound_q8 (restated here with its
1% slack). This test replays the screen's arithmetic in numpy, bit for bit
where it rounds (FP32 products, rint, floor, the single FP32 conversion), on
random, clustered and adversarial rows, and checks the bound against the
exact (f64 / integer) values; it also checks the digit ranges and the int32
headroom of the sums at the largest d the screen takes.
"""

import math

import numpy as np
import pytest

D_MAX = 16384


def bound_terms(d):
    """screen_bound_q8: (e_rel, e_abs, e_min, e_lo) as the host computes them."""
    u24, u22 = 2.0 ** -24, 2.0 ** -22
    gamma = d * u24 / (1.0 - d * u24)
    rr = 0.502
    sd = math.sqrt(d)
    e_rel = np.float32((gamma + u22) * 1.01)
    e_abs = np.float32((rr * sd + u22 * 160.0 * sd) * 1.01)
    e_min = np.float32((rr * rr * d + u22 * 160.0 * 160.0 * d + 65536.0) * 1.01)
    return e_rel, e_abs, e_min, np.float32(1.01)


def quantise(m):
    """Per-row scale, integer values, digits, norm bound and low-digit norm bound."""
    m = m.astype(np.float32)
    mx = np.abs(m).max(axis=1)
    s = np.where(mx > 0, np.float32(32638.0) / np.where(mx > 0, mx, 1), np.float32(1.0))
    s = s.astype(np.float32)
    v = np.rint((m * s[:, None]).astype(np.float32)).astype(np.int64)
    hi = np.floor((v + 128) / 256).astype(np.int64)
    lo = v - 256 * hi
    nrm = (np.sqrt((m.astype(np.float64) ** 2).sum(1)) * (1 + 1 / 512)).astype(np.float32)
    lon = (np.sqrt((lo.astype(np.float64) ** 2).sum(1)) * (1 + 1 / 512)).astype(np.float32)
    return s, v, hi, lo, nrm, lon


def check(x, c):
    d = x.shape[1]
    e_rel, e_abs, e_min, e_lo = bound_terms(d)
    sx, vx, hx, lx, xn, xlo = quantise(x)
    # The centroid set shares one scale, from max |c| over all of it.
    mxc = np.float32(np.abs(c.astype(np.float32)).max())
    sc = np.float32(32638.0) / mxc if mxc > 0 else np.float32(1.0)
    wc = np.rint((c.astype(np.float32) * sc).astype(np.float32)).astype(np.int64)
    hc = np.floor((wc + 128) / 256).astype(np.int64)
    lc = wc - 256 * hc
    cmax = np.float32(np.sqrt((c.astype(np.float64) ** 2).sum(1)).max() * (1 + 1 / 512))
    clo = np.float32(np.sqrt((lc.astype(np.float64) ** 2).sum(1)).max() * (1 + 1 / 512))
    for arr, lim in ((hx, 127), (hc, 127)):
        assert arr.min() >= -lim and arr.max() <= lim
    for arr in (lx, lc):
        assert arr.min() >= -128 and arr.max() <= 127
    hh = hx @ hc.T
    mid = hx @ lc.T + lx @ hc.T
    assert np.abs(hh).max() < 2 ** 31 and np.abs(mid).max() < 2 ** 31
    a = (hh + np.floor_divide(mid, 256)).astype(np.float32).astype(np.float64)  # one conversion
    xs = (xn * sx).astype(np.float32)
    cs = np.float32(cmax * sc)
    e_acc = (e_rel * xs * cs + e_abs * (xs + cs) + e_min).astype(np.float64)
    e_acc = e_acc + float(e_lo) * xlo.astype(np.float64) * float(clo)
    # Exact scaled dot and the FP32 chain's own deviation from it.
    exact = (x.astype(np.float64) * sx[:, None].astype(np.float64)) @ (
        c.astype(np.float64) * float(sc)).T
    chain = np.empty_like(exact)
    xf, cf = x.astype(np.float32), c.astype(np.float32)
    for i in range(x.shape[0]):
        acc = np.zeros(c.shape[0], np.float32)
        for t in range(d):  # sequential FMA chain, emulated with f64 products rounded once
            acc = (acc.astype(np.float64) + xf[i, t].astype(np.float64) * cf[:, t]).astype(np.float32)
        chain[i] = acc.astype(np.float64) * float(sx[i]) * float(sc)
    # Rows whose bound is not finite (a norm past the FP32 range) are not
    # screened: the kernel sends them to the exact scan.
    screened = np.isfinite(e_acc)
    err = np.abs(65536.0 * a - exact) + np.abs(chain - exact)
    ratio = err[screened] / e_acc[screened][:, None]
    assert ratio.size == 0 or ratio.max() <= 1.0, ratio.max()
    # The screen's own part (everything but the FP32 chain's gamma_d term)
    # against its own error.
    gamma = d * 2.0 ** -24 / (1.0 - d * 2.0 ** -24) * 1.01
    e_own = e_acc - gamma * xs.astype(np.float64) * float(cs)
    own = np.abs(65536.0 * a - exact)[screened] / e_own[screened][:, None]
    assert own.size == 0 or own.max() <= 1.0, own.max()
    return screened, (own.max() if own.size else 0.0)


def rows(kind, n, d, seed):
    rng = np.random.default_rng(seed)
    if kind == "gauss":
        return rng.standard_normal((n, d)).astype(np.float32)
    if kind == "clustered":
        base = rng.standard_normal(d).astype(np.float32)
        return (base + 0.01 * rng.standard_normal((n, d))).astype(np.float32)
    if kind == "spiky":  # one large value per row, the rest tiny: coarse scales
        m = (1e-3 * rng.standard_normal((n, d))).astype(np.float32)
        m[np.arange(n), rng.integers(0, d, n)] = 50.0
        return m
    if kind == "halves":  # values at x.5 of the integer grid after scaling
        m = np.full((n, d), 0.5, np.float32)
        m[:, 0] = 32638.0
        return m * np.float32(1e-3)
    if kind == "aligned":
        # Every scaled value 0.49 above an integer whose low digit is 127, all
        # positive: the rounding errors and the dropped lo.lo products add up
        # with one sign, close to the bound's worst case.
        m = np.full((n, d), np.float32(25727.49) / np.float32(32638.0), np.float32)
        m[:, 0] = 1.0
        return m
    if kind == "large":  # large but finite norms and products
        return (rng.standard_normal((n, d)) * 1e15).astype(np.float32)
    if kind == "extreme":  # norms past the FP32 range
        return rng.choice(np.array([1.0, -1.0], np.float32), (n, d)) * np.float32(3e38)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["gauss", "clustered", "spiky", "halves", "large"])
@pytest.mark.parametrize("d", [16, 100, 768])
def test_fixed_point_bound_holds(kind, d):
    x = rows(kind, 6, d, d)
    c = rows(kind, 9, d, d + 1)
    screened, worst = check(x, c)
    assert screened.all()
    assert worst > 0.0


@pytest.mark.parametrize("d", [16, 768, 4096])
def test_fixed_point_bound_is_nearly_reached(d):
    """Coherent worst-case rows come close to the screen's own bound (so the
    check above would see a bound that is too small), and stay under it."""
    x = rows("aligned", 2, d, 0)
    c = rows("aligned", 3, d, 1)
    screened, worst = check(x, c)
    assert screened.all()
    assert 0.8 < worst <= 1.0, worst


def test_rows_past_the_fp32_range_are_not_screened():
    x = rows("extreme", 4, 64, 1)
    c = rows("gauss", 5, 64, 2)
    screened, _ = check(x, c)
    assert not screened.any()


def test_sums_fit_int32_at_the_largest_d():
    # Every digit at its extreme: the hi.hi and hi.lo + lo.hi sums at d = 16384.
    assert D_MAX * 127 * 127 < 2 ** 31
    assert D_MAX * 2 * 127 * 128 < 2 ** 31
    assert D_MAX * 127 * 127 + D_MAX * 2 * 127 * 128 // 256 + 1 < 2 ** 31
