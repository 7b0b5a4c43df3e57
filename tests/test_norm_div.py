"""The input norm's division (artlite_b200/csrc/norm.cuh div_to_f32), restated in NumPy float64 (IEEE products and
quotients, as the GPU's): float32(v / d) from one product v (1 / d), with the division itself taken near a float32
rounding boundary, equals the reference's float32(float64 v / d) (tests/np_ops.py:27-32) on random operands and on
operands built to land within a few float64 units of a float32 midpoint."""

import numpy as np


def div_to_f32(v: np.ndarray, d: np.ndarray) -> np.ndarray:
    r = 1.0 / d
    q = v * r
    b = q.view(np.uint64)
    low = (b & np.uint64(0x1FFFFFFF)).astype(np.int64)
    e = ((b >> np.uint64(52)) & np.uint64(0x7FF)).astype(np.int64)
    fast = ((np.abs(low - 0x10000000) > 4) & (e >= 1023 - 125) & (e <= 1023 + 126)) | ((b << np.uint64(1)) == 0)
    with np.errstate(all="ignore"):
        return np.where(fast, q, v / d).astype(np.float32)


def _want(v, d):
    with np.errstate(all="ignore"):
        return (v / d).astype(np.float32)


def test_random_operands():
    rng = np.random.default_rng(0)
    n = 2_000_000
    v = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32).astype(np.float64)
    d = np.sqrt(np.abs(rng.standard_normal(n)) * np.exp2(rng.integers(-30, 30, n)) + 1e-6)
    assert np.array_equal(div_to_f32(v, d).view(np.uint32), _want(v, d).view(np.uint32))


def test_near_float32_midpoints():
    """v / d placed k float64 units from a float32 midpoint (k = -40 .. 40), where the product and the quotient can
    round to different float32 values: the guard must send those to the division."""
    rng = np.random.default_rng(1)
    n = 20_000
    f = (rng.standard_normal(n) * np.exp2(rng.integers(-10, 10, n))).astype(np.float32)
    m = (f.astype(np.float64) + np.nextafter(f, np.float32(np.inf)).astype(np.float64)) / 2  # midpoints (exact)
    v = (rng.standard_normal(n) * 4).astype(np.float32).astype(np.float64)
    base = v / m
    hits = 0
    for k in range(-40, 41):
        d = base * (1.0 + k * 2.0 ** -52)
        got, want = div_to_f32(v, d), _want(v, d)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), k
        q = v * (1.0 / d)
        hits += int(np.sum(q.astype(np.float32) != want))  # where the product alone would have been wrong
    assert hits > 0  # (the construction reaches the cases the guard exists for)


def test_special_values():
    v = np.array([0.0, -0.0, 1.0, -3.0, np.inf, -np.inf, np.nan, 1e-40, 3e38, 1.0, 0.0, 1.0], np.float64)
    d = np.array([2.0, 2.0, 0.0, 0.0, 3.0, np.inf, 1.0, 1.0, 1e-3, np.inf, 0.0, 1e-300], np.float64)
    got, want = div_to_f32(v, d), _want(v, d)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
