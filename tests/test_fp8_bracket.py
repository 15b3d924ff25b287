"""The bracket behind the exact FP8 codes (afb_device.cuh e4m3_try8), in IEEE
float32 on the host.

With s = RN(amax / 448), r = RN(1 / s), rl = RN(r * (1 - 2^-22)) and
rh = RN(r * (1 + 2^-22)), the kernels convert RN(y * rl) and RN(y * rh) and
keep the code when both agree.  That is only sound if those two products
bracket the correctly rounded quotient RN(y / s) in magnitude; e4m3 rounding
is monotone, so the quotient's code then lies between theirs.  numpy's
float32 multiply and divide round to nearest even, as the device's
mul.rn / div.rn do.
"""
import numpy as np

F = np.float32


def _bracket(y: np.ndarray, amax: np.ndarray):
    s = (np.maximum(amax, F(1e-12)) / F(448.0)).astype(F)
    r = (F(1.0) / s).astype(F)
    rl = (r * F(1.0 - 2.0 ** -22)).astype(F)
    rh = (r * F(1.0 + 2.0 ** -22)).astype(F)
    return (y * rl).astype(F), (y / s).astype(F), (y * rh).astype(F)


def test_bracket_holds_over_scales():
    rng = np.random.default_rng(7)
    n = 1 << 21
    # row maxima from 1e-12 to 1e30, elements anywhere in [-amax, amax]
    amax = (10.0 ** rng.uniform(-12, 30, n)).astype(F)
    y = (amax * rng.uniform(-1, 1, n).astype(F)).astype(F)
    # tiny elements, whose quotients land near the fp32 subnormal range
    y[: n // 8] = (y[: n // 8] * F(2.0 ** -40)).astype(F)
    a, q, b = _bracket(y, amax)
    assert np.all(np.abs(a) <= np.abs(q))
    assert np.all(np.abs(q) <= np.abs(b))


def test_bracket_holds_next_to_e4m3_ties():
    """Quotients within a few fp32 steps of e4m3 rounding midpoints, where
    the bracket is the only thing deciding the code."""
    rng = np.random.default_rng(11)
    n = 1 << 20
    amax = (10.0 ** rng.uniform(-6, 6, n)).astype(F)
    s = (amax / F(448.0)).astype(F)
    # e4m3 midpoints m * 2^E with m = 8.5 .. 15.5 (normal range) or k + 0.5
    # steps of 2^-9 (subnormal range), then a few ulps either way
    E = rng.integers(-6, 8, n)
    mid = (rng.integers(8, 16, n) + 0.5) * np.exp2(E - 3.0)
    sub = rng.random(n) < 0.2
    mid[sub] = (rng.integers(0, 8, sub.sum()) + 0.5) * 2.0 ** -9
    t = mid.astype(F)
    t = (t + (rng.integers(-4, 5, n) * np.spacing(t))).astype(F)
    y = (t * s).astype(F) * np.where(rng.random(n) < 0.5, F(-1), F(1))
    a, q, b = _bracket(y.astype(F), amax)
    assert np.all(np.abs(a) <= np.abs(q))
    assert np.all(np.abs(q) <= np.abs(b))
