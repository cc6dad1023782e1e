"""CPU: property tests of the oracle's building blocks against independent
brute-force formulations (hypothesis-generated inputs, exact rounding ties
and range edges included).  The pins in test_oracle_pins.py check the same
functions against the reference at fixed points; these check the rules
themselves over many inputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.extra import numpy as hnp  # noqa: E402

from oracle import h3_oracle as O  # noqa: E402

SETTINGS = settings(max_examples=150, deadline=None)
E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
# every e2m1 midpoint and every e4m3 midpoint, so ties are drawn often
E2M1_TIES = [(a + b) / 2 for a, b in zip(E2M1_MAG[:-1], E2M1_MAG[1:])]
E4M3_POS = O.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8)).astype(np.float64)
E4M3_TIES = list(((E4M3_POS[:-1] + E4M3_POS[1:]) / 2).astype(np.float32))


def _nearest_even(v: float, table: np.ndarray) -> int:
    """Index of the value of `table` (ascending) nearest to v; a tie goes to
    the even index (even mantissa); beyond the last value, the last index."""
    d = np.abs(table - v)
    best = np.flatnonzero(d == d.min())
    return int(best[0] if len(best) == 1 else best[best % 2 == 0][0])


f32 = st.floats(allow_nan=False, allow_infinity=False, width=32)


@SETTINGS
@given(st.lists(st.one_of(f32, st.sampled_from(E2M1_TIES + [-t for t in E2M1_TIES] + [0.0, -0.0, 6.0, 7.5])),
                min_size=1, max_size=64))
def test_e2m1_is_round_half_even_with_saturation(vals):
    r = np.array(vals, dtype=np.float32)
    got = O.e2m1_rne_sat(r)
    for v, code in zip(r, got):
        mag = _nearest_even(min(abs(float(v)), 6.0), E2M1_MAG)
        assert int(code) == mag | (int(np.signbit(v)) << 3), (v, code)


@SETTINGS
@given(st.lists(st.one_of(st.floats(min_value=0.0, max_value=1e6, width=32), st.sampled_from(E4M3_TIES),
                          st.sampled_from([0.0, 2.0 ** -9, 2.0 ** -10, 448.0, 464.0, 480.0])),
                min_size=1, max_size=64))
def test_e4m3_is_round_half_even_with_saturation(vals):
    v = np.array(vals, dtype=np.float32)
    got = O.e4m3_rn_satfinite(v)
    for x, code in zip(v, got):
        assert int(code) == _nearest_even(min(float(x), 448.0), E4M3_POS), (x, code)


@SETTINGS
@given(st.integers(1, 300), st.integers(1, 40), st.integers(0, 2 ** 31))
def test_blocked_layout_round_trip(rows, ncols, seed):
    rng = np.random.default_rng(seed)
    sf = rng.integers(1, 256, (rows, ncols), dtype=np.uint8)
    flat = O.to_blocked(sf)
    assert flat.size == (rows + 127) // 128 * 128 * ((ncols + 3) // 4 * 4)
    assert np.array_equal(O.from_blocked(flat, rows, ncols), sf)
    r, c = np.meshgrid(np.arange(rows), np.arange(ncols), indexing="ij")
    off = O.blocked_offset(r, c, ncols).ravel()
    assert len(np.unique(off)) == off.size  # a bijection onto the stored positions
    pad = np.ones(flat.size, dtype=bool)
    pad[off] = False
    assert not flat[pad].any()  # padding rows and columns are zero


@SETTINGS
@given(hnp.arrays(np.float32, st.tuples(st.integers(1, 6), st.integers(1, 96)),
                  elements=st.floats(-1e4, 1e4, width=32)))
def test_int8_rows_stay_in_range_and_within_half_a_step(x):
    q, s = O.dynamic_quant_rows(torch.from_numpy(x))
    qn, sn = q.numpy().astype(np.float64), s.numpy().astype(np.float64)
    assert np.abs(qn).max() <= 127
    err = np.abs(x.astype(np.float64) - qn * sn[:, None])
    # half a step, plus the fp32 rounding of x / scale
    assert (err <= sn[:, None] * (0.5 + 1e-5) + 1e-30).all()


@SETTINGS
@given(hnp.arrays(np.uint8, st.integers(0, 256)))
def test_swap_nibbles_is_an_involution(b):
    t = torch.from_numpy(b)
    once = O.swap_nibbles(t)
    assert torch.equal(O.swap_nibbles(once), t)
    assert torch.equal(once & 0xF, t >> 4) and torch.equal(once >> 4, t & 0xF)
