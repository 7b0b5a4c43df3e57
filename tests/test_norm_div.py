"""The input norm's division (artlite_b200/csrc/norm.cuh div_to_f32), restated in Python with exact fused
multiply-adds (fractions, rounded once to float64): float32(v / d) from the reciprocal r = 1 / d by a product and two
FMA-remainder corrections equals the reference's float32(float64 v / d) (tests/np_ops.py:27-32) bit for bit, on
random operands and on operands built to land within a few float64 units of a float32 midpoint."""

from fractions import Fraction

import numpy as np


def _fma(a: float, b: float, c: float) -> float:
    return float(Fraction(a) * Fraction(b) + Fraction(c))  # (int / int division: correctly rounded)


def div_to_f32(v: float, d: float) -> np.float32:
    r = 1.0 / d
    q0 = v * r
    q1 = _fma(_fma(-q0, d, v), r, q0)
    q2 = _fma(_fma(-q1, d, v), r, q1)
    return np.float32(q2 if q2 != 0.0 else q0)


def _check(vs, ds):
    for v, d in zip(vs, ds):
        got, want = div_to_f32(float(v), float(d)), np.float32(float(v) / float(d))
        assert got.view(np.uint32) == want.view(np.uint32), (v, d)


def test_random_operands():
    rng = np.random.default_rng(0)
    n = 6000
    v = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32).astype(np.float64)
    d = np.sqrt(np.abs(rng.standard_normal(n)) * np.exp2(rng.integers(-30, 30, n)) + 1e-6)
    _check(v, d)


def test_near_float32_midpoints():
    """v / d placed k float64 units from a float32 midpoint (k = -40 .. 40), where a product alone can round to the
    other float32 neighbour."""
    rng = np.random.default_rng(1)
    n = 120
    f = (rng.standard_normal(n) * np.exp2(rng.integers(-10, 10, n))).astype(np.float32)
    m = (f.astype(np.float64) + np.nextafter(f, np.float32(np.inf)).astype(np.float64)) / 2  # midpoints (exact)
    v = (rng.standard_normal(n) * 4).astype(np.float32).astype(np.float64)
    off = 0
    for k in range(-40, 41):
        d = v / m * (1.0 + k * 2.0 ** -52)
        _check(v, d)
        off += int(np.sum((v * (1.0 / d)).astype(np.float32) != (v / d).astype(np.float32)))
    assert off > 0  # (the construction reaches cases a single product gets wrong)


def test_signed_zero_and_extremes():
    v = np.array([0.0, -0.0, 3.0e38, -1.0e-38, 1.401298464324817e-45, 1.0], np.float64)
    d = np.array([2.0, -2.0, 1.0e-3, 7.0, 3.0, 2.0 ** -149], np.float64)
    _check(v, d)
