"""CPU: pin the oracle restatement against the reference's own Python and the
committed golden fixtures (generated from the reference by
tests/golden/make_golden.py)."""
from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import load_golden
from oracle import h3_oracle as O


def _outliers(seed: int, m: int, k: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    return torch.where(torch.rand(m, k, generator=g) < 0.001, 20 * x, x).to(torch.bfloat16)


# ---------------------------------------------------------------- INT8

def test_int8_quant_matches_reference(ref):
    for seed, (m, k) in enumerate([(7, 3072), (33, 12288), (5, 8)]):
        x = _outliers(seed, m, k)
        q_ref, s_ref = ref.int8_convrot._dynamic_quant_rows(x)
        q, s = O.dynamic_quant_rows(x)
        assert torch.equal(q, q_ref) and torch.equal(s, s_ref)


def test_int8_quant_golden():
    g = load_golden("int8_quant.pt")
    q, s = O.dynamic_quant_rows(g["x"])
    assert torch.equal(q, g["q"]) and torch.equal(s, g["scale"])
    assert (g["q"][-2] == 0).all() and (g["q"][-1] == 0).all()  # zero row, tiny row (1e-12 clamp)


def test_int8_acc_exact():
    g = torch.Generator().manual_seed(3)
    q = torch.randint(-128, 128, (17, 256), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (40, 256), generator=g, dtype=torch.int8)
    want = (q.to(torch.int64) @ w.to(torch.int64).T).to(torch.int32)
    assert torch.equal(O.int8_acc(q, w), want)
    assert torch.equal(O.int8_acc(q, w), torch._int_mm(q.contiguous(), w.T.contiguous()))


# ---------------------------------------------------------------- NVFP4

def test_e4m3_decode_matches_reference(ref):
    bits = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    want = ref.float8_cast._fp8_e4m3fn_to_f32(bits).numpy()
    got = O.e4m3_decode(bits.numpy())
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok], want[ok])


def test_e4m3_encoder_is_round_nearest_even():
    rng = np.random.default_rng(0)
    v = np.abs(rng.standard_normal(100_000).astype(np.float32)) * np.float32(60)
    mids = ((O._E4M3_POS[1:] + O._E4M3_POS[:-1]) / 2).astype(np.float32)
    v = np.concatenate([v, O._E4M3_POS, mids, np.float32([0, 1e-9, 447, 448, 464, 1e6])]).astype(np.float32)
    want = torch.from_numpy(np.minimum(v, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_rn_satfinite(v), want)


def test_blocked_layout_matches_reference(ref):
    g = torch.Generator().manual_seed(5)
    for rows, ncols in [(130, 16), (256, 192), (7, 4)]:
        sf = torch.randint(0, 127, (rows, ncols), generator=g, dtype=torch.uint8)
        flat = torch.from_numpy(O.to_blocked(sf.numpy()))
        padded = flat.reshape((rows + 127) // 128 * 128, (ncols + 3) // 4 * 4)
        assert torch.equal(ref.nvfp4.from_blocked(padded, rows, ncols), sf)


def test_nvfp4_roundtrip_through_reference_decode(ref):
    x = _outliers(11, 200, 512)
    qz = O.nvfp4_quantize(x, hi_first=True)
    want = ref.nvfp4.dequantize_nvfp4(qz["codes"], qz["gs"], qz["sf"].view(torch.float8_e4m3fn),
                                      out_dtype=torch.float32)
    got = O.nvfp4_dequantize(qz["codes"], qz["gs"], qz["sf"], 512, hi_first=True)
    assert torch.equal(got, want)
    # quantisation error is bounded by half an e2m1 step of each block's scale
    assert (got - x.float()).abs().max() <= x.float().abs().max() / 6 * 1.01


def test_nvfp4_golden():
    g = load_golden("nvfp4.pt")
    qz = O.nvfp4_quantize(g["x"], hi_first=True)
    assert torch.equal(qz["codes"], g["codes_hi_first"])
    assert torch.equal(qz["sf"], g["sf"]) and torch.equal(qz["gs"], g["gs"])
    k = g["x"].shape[1]
    assert torch.equal(O.nvfp4_dequantize(qz["codes"], qz["gs"], qz["sf"], k), g["dequant_f32"])
    lo = O.nvfp4_quantize(g["x"], hi_first=False)
    assert torch.equal(O.swap_nibbles(lo["codes"]), g["codes_hi_first"])


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vllm not installed")
def test_nvfp4_quantiser_vs_independent_implementation():
    """The reference's own NVFP4 quantiser is not in its sources, so the
    oracle's is compared with an independent one, vllm's pure-torch
    ref_nvfp4_quant (run in a child process by nvfp4_vllm_xcheck.py).  The
    two must agree on every block scale and code except at exact rounding
    ties, where the recipes' different fp32 orders (divide vs multiply by a
    reciprocal) decide; there they may differ by one step.  The weights case
    is built to contain such ties, so that path is exercised."""
    script = Path(__file__).with_name("nvfp4_vllm_xcheck.py")
    out = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    result = json.loads(out.stdout.strip().splitlines()[-1])
    for name, c in result.items():
        assert c["scale_tie_dist_max"] == 0.0 and c["code_tie_dist_max"] == 0.0, (name, c)
        assert c["scale_steps_apart_max"] <= 1, (name, c)
        assert c["scale_mismatches"] <= 0.02 * c["scales"], (name, c)
        assert c["code_mismatches"] <= 0.002 * c["codes_compared"], (name, c)
    assert result["weights"]["scale_mismatches"] > 0


def test_nvfp4_row_group_sampling():
    """The full-size GPU checks quantise only sampled 128-row groups on the
    CPU.  That equals slicing the whole tensor's quantisation when the group
    holding the global max is among them, and each group's blocked scales
    are one contiguous chunk of (k/16 rounded up to 4) * 128 bytes."""
    gen = torch.Generator().manual_seed(5)
    m, k = 640, 208  # k/16 = 13 scale columns: the last 4-column block is padded
    x = torch.randn(m, k, generator=gen)
    x[130, 17] = 50.0
    full = O.nvfp4_quantize(x.to(torch.bfloat16), hi_first=False)
    groups = [1, 3]
    rows = torch.cat([torch.arange(g * 128, g * 128 + 128) for g in groups])
    part = O.nvfp4_quantize(x[rows].to(torch.bfloat16), hi_first=False)
    chunk = (k // 16 + 3) // 4 * 512
    assert torch.equal(part["gs"], full["gs"])
    assert torch.equal(part["codes"], full["codes"][rows])
    assert torch.equal(part["sf"], torch.cat([full["sf"][g * chunk:(g + 1) * chunk] for g in groups]))


# ---------------------------------------------------------------- RoPE / norm

def test_rope_golden():
    g = load_golden("rope.pt")
    angles = O.rope_angles(g["pos"], g["inv_freq"], g["n_t"], g["n_h"])
    table = O.rope_rotation_table(angles, torch.bfloat16)
    assert torch.equal(table, g["table"])
    out = O.rms_rope_apply(g["q"], table, g["weight"], g["eps"], 128)
    assert torch.equal(out, g["out"])


def test_rope_matches_reference(ref):
    g = torch.Generator().manual_seed(8)
    pos = O.grid_positions(3, 4, 5)
    x = torch.randn(1, 60, 2, 128, generator=g).to(torch.bfloat16)
    w = torch.ones(128, dtype=torch.bfloat16)
    angles = O.rope_angles(pos, O.rope_inv_freq(), 22, 21)
    t_ref = ref.rope.rope_rotation_table(angles, torch.bfloat16)
    assert torch.equal(O.rope_rotation_table(angles, torch.bfloat16), t_ref)
    assert torch.equal(O.rms_rope_apply(x, t_ref, w, 1e-6, 128), ref.rope.rms_rope_apply(x, t_ref, w, 1e-6, 128))
    assert torch.equal(O.rms_norm(x, w, 1e-5), ref.linear.RMSNorm(128, eps=1e-5)(x))


# ---------------------------------------------------------------- attention / block

def test_attention_golden():
    g = load_golden("attention.pt")
    o = O.attention_fp32(g["q"][0], g["k"][0], g["v"][0])
    assert (o - g["out"][0].float()).abs().max() < 2e-2


def test_ulysses_layout_matches_reference_permutation():
    """seq->head: rank r receives every rank's tokens (rank order) for heads
    [r*H/ws, (r+1)*H/ws) — ops/ulysses.py:28-31 evaluated for all ranks."""
    ws, s_local, h, d = 4, 3, 8, 2
    full = torch.arange(ws * s_local * h * d, dtype=torch.float32).reshape(ws * s_local, h, d)
    shards = full.chunk(ws, dim=0)
    sends = [x.view(s_local, ws, h // ws, d).permute(1, 0, 2, 3).contiguous() for x in shards]
    for r in range(ws):
        recv = torch.stack([sends[src][r] for src in range(ws)])  # all_to_all_single
        got = recv.reshape(ws * s_local, h // ws, d)
        assert torch.equal(got, O.seq_to_head_local(full, ws, r))


def _block_linear(params, fmt):
    lin = {n: O.EmulatedQuantLinear(params[f"{n}_w"], fmt) for n in ("qkv", "out", "fc1", "fc2")}
    return lambda name, x: lin[name](x)


def test_dit_block_golden_bit_exact():
    from golden.make_golden import block_fixture_params

    for name in ("dit_block_int8_gelu.pt", "dit_block_nvfp4_gelu.pt", "dit_block_nvfp4_swiglu.pt"):
        g = load_golden(name)
        params = block_fixture_params(g)
        out = O.dit_block_forward(g["x"].clone(), g["t_emb"], g["segments"], params, heads=g["heads"],
                                  head_dim=128, eps=g["eps"], qk_eps=g["qk_eps"], mlp_act=g["mlp_act"],
                                  pos=g["pos"], inv_freq=g["inv_freq"], n_t=g["n_t"], n_h=g["n_h"],
                                  linear=_block_linear(params, g["fmt"]), attn_fp32=False)
        assert torch.equal(out, g["out"]), name


# ---------------------------------------------------------------- ConvRot

def test_hadamard_matrix_matches_reference(ref):
    for size in (4, 16, 64, 256):
        h_ref = ref.hadamard.build_hadamard(size, torch.device("cpu"), torch.float64).numpy()
        assert np.array_equal(O.hadamard_matrix(size), h_ref)


def test_rotation_matches_reference(ref):
    """The exact, singly rounded rotation against the reference's 16-bit
    torch.mm: identical for bf16; for fp16 the reference's CPU GEMM is not
    correctly rounded in a few elements (at most 2 ulp)."""
    x = _outliers(11, 64, 3072)
    for dt, max_ulp, max_frac in ((torch.bfloat16, 0, 0.0), (torch.float16, 2, 2e-4)):
        xd = x.to(dt)
        a = O.rotate_activation_exact(xd, 256)
        b = ref.hadamard.rotate_activation(xd, 256)
        ulp = (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()
        assert int(ulp.max()) <= max_ulp
        assert (ulp > 0).float().mean().item() <= max_frac


def test_convrot_golden():
    g = load_golden("convrot.pt")
    for name, max_ulp in (("bf16", 0), ("f16", 2)):
        rot = O.rotate_activation_exact(g[f"x_{name}"], 256)
        ulp = (rot.view(torch.int16).int() - g[f"rot_{name}"].view(torch.int16).int()).abs()
        assert int(ulp.max()) <= max_ulp
    # bf16: rotation and row quantisation bit-exact to the reference's
    q, s = O.dynamic_quant_rows(O.rotate_activation_exact(g["x_bf16"], 256))
    assert torch.equal(q, g["q_bf16"]) and torch.equal(s, g["scale_bf16"])


def test_rotation_is_orthonormal():
    h = O.hadamard_matrix(256)
    assert np.allclose(h @ h.T, np.eye(256), atol=1e-12)
