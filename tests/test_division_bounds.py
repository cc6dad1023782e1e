"""CPU: the bound behind the quantisers' per-row / per-block range check.

The INT8 and NVFP4 kernels divide every element by its row or block divisor
b as Markstein's corrected quotient from y = RN(1/b):

    q0 = RN(a * y);  r = RN(a - q0 * b) (one FMA);  q = RN(q0 + r * y) (one FMA)

which is the correctly rounded a / b unless the residual underflows, i.e.
for |a| < 2^-90.  The kernels skip the per-element test whenever
2^-86 <= b <= 2^96, relying on this: for such b and |a| < 2^-90, |q| stays
below 1/4, so the INT8 code (rint) and the e2m1 code (RNE, 1/4 rounds to 0)
are zero exactly as for the true quotient; and copysign(q, a) carries the
sign of a, which the e2m1 code keeps (a -0 dividend alone comes out +0).
Here the FMAs are emulated exactly: the product of two fp32 values is exact
in fp64 and the sum is rounded once to fp32.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _fma32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def _markstein(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    # quotients that overflow fp32 end as inf / nan here; callers drop them
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        y = (F32(1) / b).astype(np.float32)
        q0 = (a * y).astype(np.float32)
        r = _fma32(-q0, b, a)
        return _fma32(r, y, q0)


def _tiny_bf16_dividends(rng: np.random.Generator, n: int) -> np.ndarray:
    """bf16-representable values below 2^-90 in magnitude (subnormals
    included) with both signs, plus signed zeros and the extremes."""
    e = rng.integers(-133, -90, n)
    m = rng.integers(0, 128, n)
    a = (np.ldexp(1 + m / 128.0, e) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
    edge = np.float32([0.0, -0.0, 2.0 ** -133, -(2.0 ** -133), np.nextafter(F32(2.0 ** -90), F32(0))])
    return np.concatenate([a, edge]).astype(np.float32)


def test_tiny_dividends_give_zero_codes_with_their_sign():
    rng = np.random.default_rng(0)
    a = _tiny_bf16_dividends(rng, 100_000)
    for be in range(-86, 97):
        b = np.full_like(a, F32(np.ldexp(1.0 + rng.random(), be)))
        q = _markstein(a, b)
        assert (np.abs(q) < 0.25).all(), be
        assert (np.signbit(np.copysign(q, a)) == np.signbit(a)).all(), be
    # the lower end exactly
    b = np.full_like(a, F32(2.0 ** -86))
    assert (np.abs(_markstein(a, b)) < 0.25).all()


def test_markstein_is_the_correctly_rounded_quotient_above_the_guard():
    """Where the per-element test used to send elements (|a| >= 2^-90), the
    corrected quotient equals the IEEE quotient RN(a / b)."""
    rng = np.random.default_rng(1)
    n = 200_000
    a = (np.ldexp(1 + rng.integers(0, 128, n) / 128.0, rng.integers(-90, 120, n))
         * rng.choice([-1.0, 1.0], n)).astype(np.float32)
    b = np.ldexp(1.0 + rng.random(n), rng.integers(-86, 96, n)).astype(np.float32)
    q = _markstein(a, b)
    with np.errstate(over="ignore", under="ignore"):
        exact = (a.astype(np.float64) / b.astype(np.float64)).astype(np.float32)
    finite = np.isfinite(exact) & (np.abs(exact) >= np.finfo(np.float32).tiny)
    assert np.array_equal(q[finite], exact[finite])
