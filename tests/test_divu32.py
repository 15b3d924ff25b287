"""The division by a launch-constant divisor that the kernels use for
row -> batch entry and token -> position (DivU32 in afb_device.cuh):
Granlund and Montgomery's multiply-high method, checked here over its whole
parameter domain on restated integer arithmetic.  The device code itself is
covered by the GPU parity tests, whose shapes put rows of several batch
entries (odd sequence lengths) in one CTA."""
import numpy as np


def make_divu32(d):
    """m, s1, s2, wide for divisor d, as make_divu32() forms them."""
    d = max(d, 1)
    if d > 1 << 32:
        return 0, 0, 0, True
    l = 0
    while (1 << l) < d:
        l += 1
    m = ((1 << 32) * ((1 << l) - d)) // d + 1
    assert m < 1 << 32
    return m, min(l, 1), max(l - 1, 0), False


def div_u32(params, d, n):
    """q = n // d as div_u32() forms it for 0 <= n < 2^32 (uint32 lanes)."""
    m, s1, s2, wide = params
    if wide:
        return n // d
    n = np.asarray(n, dtype=np.uint64)
    t = (n * np.uint64(m)) >> np.uint64(32)
    return (t + ((n - t) >> np.uint64(s1))) >> np.uint64(s2)


def _dividends(rng):
    edge = np.array([0, 1, 2, 3, (1 << 31) - 1, 1 << 31, (1 << 32) - 2, (1 << 32) - 1], dtype=np.uint64)
    return np.concatenate([edge, np.arange(0, 70000, dtype=np.uint64),
                           rng.integers(0, 1 << 32, size=20000, dtype=np.uint64)])


def test_divu32_small_divisors():
    rng = np.random.default_rng(7)
    n = _dividends(rng)
    for d in range(1, 1200):
        q = div_u32(make_divu32(d), d, n)
        assert np.array_equal(q, n // np.uint64(d)), d


def test_divu32_large_and_edge_divisors():
    rng = np.random.default_rng(8)
    n = _dividends(rng)
    ds = [4096, 4097, 8191, 9000, 33000, 65535, 65537, (1 << 31) - 1, 1 << 31, (1 << 31) + 1,
          (1 << 32) - 1, 1 << 32]
    ds += [1 << k for k in range(33)] + [(1 << k) + 1 for k in range(1, 32)] + [(1 << k) - 1 for k in range(2, 33)]
    ds += [int(x) for x in rng.integers(2, 1 << 32, size=200)]
    for d in ds:
        q = div_u32(make_divu32(d), d, n)
        assert np.array_equal(q, n // np.uint64(d)), d


def test_divu32_wide_divisor_takes_the_division():
    p = make_divu32((1 << 32) + 5)
    assert p[3]
    assert div_u32(p, (1 << 32) + 5, 1 << 40) == (1 << 40) // ((1 << 32) + 5)
