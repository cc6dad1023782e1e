"""CPU checks of the arithmetic facts the packed row kernels rely on.

* The reference computes each bf16 step of RMSNorm + modulate and of RoPE as
  an fp32 operation rounded to bf16 (bf16(fp32(a) op fp32(b))).  The kernels
  run those steps on `mul.rn.bf16x2` / `add.rn.bf16x2`, which round the exact
  result to bf16 once.  For two bf16 operands the two agree: a product of two
  8-bit significands is exact in fp32, and a sum is either exact in fp32 or
  its smaller operand is too small to move the bf16 result.
* The INT8 quantisers take rint(q) for |q| <= 127 (1 + 2^-23) from the low
  byte of fp32(q + 1.5 * 2^23): the add rounds q to an integer, ties to even.

Both are checked here on random and adversarial values with numpy, whose
float32 operations and `rint` round to nearest even; the exact values come
from float64, where every product and sum below is exact.
"""
from __future__ import annotations

import numpy as np


def _round_sig(x: np.ndarray, bits: int) -> np.ndarray:
    """Round finite, normal x to `bits` significant bits, ties to even (exact
    in float64 for the magnitudes used here)."""
    m, e = np.frexp(x)  # x = m * 2**e, 0.5 <= |m| < 1
    return np.ldexp(np.rint(m * 2.0 ** bits) / 2.0 ** bits, e)


def _bf16(x: np.ndarray) -> np.ndarray:
    return _round_sig(x, 8)


def _rand_bf16(rng: np.random.Generator, n: int, emin: int, emax: int) -> np.ndarray:
    sig = rng.integers(128, 256, n).astype(np.float64) / 256.0  # 8 significant bits
    sign = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    return sign * np.ldexp(sig, rng.integers(emin, emax + 1, n))


def _via_fp32(exact: np.ndarray) -> np.ndarray:
    """bf16(fp32(exact)): fp32 rounding first, as the reference does."""
    return _bf16(exact.astype(np.float32).astype(np.float64))


def test_bf16_product_single_rounding_matches_fp32_then_bf16():
    rng = np.random.default_rng(0)
    a = _rand_bf16(rng, 1 << 21, -30, 30)
    b = _rand_bf16(rng, 1 << 21, -30, 30)
    exact = a * b  # 16 significant bits: exact in float64 and in fp32
    assert np.array_equal(_bf16(exact), _via_fp32(exact))


def test_bf16_sum_single_rounding_matches_fp32_then_bf16():
    rng = np.random.default_rng(1)
    n = 1 << 21
    a = _rand_bf16(rng, n, -20, 20)
    # exponent gaps from 0 to 40 cover sums exact in fp32 (gap <= 16) and the
    # ones fp32 rounds (gap > 16)
    b = _bf16(_rand_bf16(rng, n, 0, 0) * np.ldexp(1.0, rng.integers(-40, 1, n)) * np.abs(a))
    for x, y in ((a, b), (b, a), (a, -b)):
        exact = x + y  # exact in float64 (gap <= 40 + 8 bits)
        nz = exact != 0
        assert np.array_equal(_bf16(exact[nz]), _via_fp32(exact[nz]))


def test_one_plus_scale_ties_and_tiny_addends():
    """bf16 addends at and around half an ulp of the other operand (exact
    ties, one step either side) and far below it (where fp32 rounds the sum
    before the bf16 rounding), and 1 + scale as in the modulation."""
    rng = np.random.default_rng(2)
    a = _rand_bf16(rng, 1 << 18, -4, 4)
    ulp = np.ldexp(1.0, np.frexp(a)[1] - 8)  # bf16 ulp of a
    addends = [ulp / 2, -ulp / 2, ulp / 2 * (1 + 2.0 ** -7), ulp / 2 * (1 - 2.0 ** -8)]
    addends += [s * ulp * 2.0 ** -k for k in range(9, 41) for s in (1.0, -1.0)]
    for y in addends:
        y = _bf16(y)
        exact = a + y
        nz = exact != 0
        assert np.array_equal(_bf16(exact[nz]), _via_fp32(exact[nz]))
    one = np.ones(1 << 18)
    sc = _rand_bf16(rng, 1 << 18, -40, 3)
    assert np.array_equal(_bf16(one + sc), _via_fp32(one + sc))


def test_rounding_add_gives_rint_in_low_byte():
    rng = np.random.default_rng(3)
    q = np.concatenate([
        rng.uniform(-127.5, 127.5, 1 << 20),
        np.arange(-127, 128) + 0.5,          # ties: to even
        np.arange(-127, 128) - 0.5,
        np.arange(-127, 128).astype(np.float64),
        np.float32(127.0) * (1 + np.float32(2.0 ** -23)) * np.array([1.0, -1.0]),
        np.array([0.0, -0.0, 2.0 ** -30, -(2.0 ** -30)]),
    ]).astype(np.float32)
    magic = np.float32(1.5 * 2 ** 23)
    t = (q + magic).astype(np.float32)
    low = (t.view(np.uint32) & 0xFF).astype(np.uint8).view(np.int8)
    want = np.rint(q).astype(np.int8)
    assert np.array_equal(low, want)


def test_int8_quotient_bound():
    """|x / s| <= 127 (1 + 2^-23) for |x| <= amax and s = fp32(amax / 127),
    so rint(x / s) never leaves [-127, 127] and the clamp does not bind."""
    rng = np.random.default_rng(4)
    amax = np.ldexp(rng.uniform(0.5, 1.0, 1 << 20), rng.integers(-40, 40, 1 << 20)).astype(np.float32)
    s = (amax.astype(np.float64) / 127.0).astype(np.float32)
    ratio = amax.astype(np.float64) / s.astype(np.float64)
    assert ratio.max() <= 127.0 * (1 + 2.0 ** -23)
    q = (amax / s).astype(np.float32)  # fp32 quotient, correctly rounded
    assert np.abs(np.rint(q)).max() <= 127
