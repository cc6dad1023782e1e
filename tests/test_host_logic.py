"""CPU: host-side layout logic of the package (no kernels launched)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import h3_oracle as O


def test_swiglu_interleave_perm_pairs_gate_and_up():
    from minixmax_h3_b200 import ops

    n = 2 * 192
    perm = ops.swiglu_interleave_perm(n)
    assert sorted(perm.tolist()) == list(range(n))
    ffn = n // 2
    for b in range(ffn // 32):
        for j in range(32):
            assert perm[64 * b + j] == 32 * b + j              # gate column 32b+j
            assert perm[64 * b + 32 + j] == ffn + 32 * b + j   # its up column


def test_permute_blocked_rows_matches_dense_permutation():
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(0)
    rows, k = 320, 512  # 3 row blocks (last one padded), 32 scale columns
    w = (torch.randn(rows, k, generator=g) * 0.02).to(torch.bfloat16)
    qz = O.nvfp4_quantize(w, hi_first=True)
    perm = ops.swiglu_interleave_perm(rows)
    out = ops.permute_blocked_rows(qz["sf"], rows, k, perm)
    dense = O.from_blocked(qz["sf"].numpy(), rows, k // 16)
    want = O.to_blocked(dense[perm.numpy()])
    assert np.array_equal(out.numpy().reshape(-1), np.asarray(want).reshape(-1))


def test_quantized_rows_must_match_the_layer():
    """INT8 rows quantised ahead of a layer (QuantizedRows, e.g. from the fused
    norm + quantise kernel) must carry the layer's ConvRot grouping; NVFP4
    layers refuse them.  Both are host-side checks."""
    import torch

    from minixmax_h3_b200.modules import QuantizedRows, QuantLinear

    w = torch.zeros(64, 256, dtype=torch.int8)
    ql = QuantLinear.from_quant_tensors(w, meta={"format": "int8_tensorwise", "convrot": True},
                                        weight_scale=torch.ones(64), device="cpu")
    rows = QuantizedRows(torch.zeros(4, 256, dtype=torch.int8), torch.ones(4), convrot_group=0)
    with pytest.raises(ValueError):
        ql._quant_i8_input(rows)
    ok = QuantizedRows(rows.q, rows.scale, convrot_group=256)
    q, s = ql._quant_i8_input(ok)
    assert q is ok.q and s is ok.scale
    assert ok.shape == (4, 256) and ok.device.type == "cpu"


def test_pre_quant_scale_applies_on_every_entry():
    """A checkpoint's pre_quant_scale multiplies the layer input before it is
    quantised (modules/linear.py:184-185) on the block's entries too: the
    input is scaled, a producer's amax of the unscaled input is dropped, and
    rows that arrive already quantised are refused.  Without the scale the
    input and amax pass through untouched."""
    import torch

    from minixmax_h3_b200.modules import QuantizedRows, QuantLinear

    w = torch.zeros(64, 256, dtype=torch.int8)
    ql = QuantLinear.from_quant_tensors(w, meta={"format": "int8_tensorwise"}, weight_scale=torch.ones(64),
                                        device="cpu")
    x = torch.randn(4, 256).to(torch.bfloat16)
    amax = torch.ones(1)
    same, same_amax = ql._pre_scale(x, amax)
    assert same is x and same_amax is amax

    pqs = torch.linspace(0.5, 2.0, 256)
    ql = QuantLinear.from_quant_tensors(w, meta={"format": "int8_tensorwise"}, weight_scale=torch.ones(64),
                                        pre_quant_scale=pqs, device="cpu")
    scaled, dropped = ql._pre_scale(x, amax)
    assert dropped is None
    assert torch.equal(scaled, x * pqs.to(torch.bfloat16))
    with pytest.raises(ValueError):
        ql._pre_scale(QuantizedRows(torch.zeros(4, 256, dtype=torch.int8), torch.ones(4)), None)


def test_ring_attention_single_process_is_one_merge_step():
    """Without a process group the ring runs one step: the chunk result is
    both the first and the last merge (it initialises and finishes the fp32
    accumulator in one call) — with the oracle's attention and merge plugged in
    it equals attention over the local keys."""
    import torch

    from minixmax_h3_b200 import ulysses as U

    calls = []

    def attn(q_, k_, v_, sc, o_, lse_):
        o, lse = O.attention_lse_fp32(q_, k_, v_, sc)
        o_.copy_(o.to(torch.bfloat16))
        lse_.copy_(lse)

    def merge(acc, acc_lse, blk, blk_lse, first, out=None, amax_out=None):
        calls.append((first, out is not None))
        acc.copy_(blk.float())
        acc_lse.copy_(blk_lse)
        if out is not None:
            out.copy_(acc.to(torch.bfloat16))

    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(40, 2, 16, generator=g).to(torch.bfloat16) for _ in range(3))
    got = U.ring_attention(q, k, v, attention_fn=attn, merge_fn=merge)
    want, _ = O.attention_lse_fp32(q, k, v)
    assert calls == [(True, True)]
    assert torch.equal(got, want.to(torch.bfloat16))


def test_no_alloc_gpu_tests_are_collected_last():
    """The allocation-free entry point's GPU tests run after every other GPU
    test, so a run that stops at the first failure has already run the
    rest: no test file may sort after tests/test_zz_no_alloc.py."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    out = subprocess.run([sys.executable, "-m", "pytest", "tests", "--collect-only", "-q", "-m", "gpu"],
                         capture_output=True, text=True, timeout=300, cwd=root)
    ids = [ln for ln in out.stdout.splitlines() if "::" in ln]
    assert ids, out.stdout[-2000:] + out.stderr[-2000:]
    files = [i.split("::")[0] for i in ids]
    first = files.index("tests/test_zz_no_alloc.py")
    assert set(files[first:]) == {"tests/test_zz_no_alloc.py"}, files[first:]


def test_curve_t_embedding_interpolates_the_table():
    """model/dit.py:870-874: t in [0, 1] -> linear interpolation between the
    two table rows around t * (grid - 1); t = 1 gives the last row exactly and
    values outside [0, 1] are clamped.  Checked against fp64 arithmetic."""
    from minixmax_h3_b200.block import curve_t_embedding

    g = torch.Generator().manual_seed(2)
    table = torch.randn(1025, 8, generator=g)
    t = torch.tensor([0.0, 1.0, 0.5, 1 / 1024, 0.3, 0.999, -0.2, 1.7])
    got = curve_t_embedding(table, t)
    assert got.shape == (8, 8) and got.dtype == torch.float32
    pos = t.double().clamp(0, 1) * 1024
    lo = pos.floor().long().clamp(max=1023)
    frac = (pos - lo).unsqueeze(1)
    want = table.double()[lo] * (1 - frac) + table.double()[lo + 1] * frac
    assert torch.allclose(got.double(), want, rtol=0, atol=1e-6)
    assert torch.equal(got[1], table[-1]) and torch.equal(got[0], table[0])
    assert torch.equal(got[6], table[0]) and torch.equal(got[7], table[-1])
    with pytest.raises(ValueError):
        curve_t_embedding(torch.zeros(1, 8), t)


def test_reference_named_int8_entries(monkeypatch):
    """ops.int8_convrot_linear / ops.rotate_activation (ops/int8_convrot.py:
    114-209, ops/hadamard.py:35-44) hand the reference's arguments to the
    quantiser and GEMM wrappers: leading dims flattened and restored, x cast
    to bf16, ConvRot group passed, scales and bias converted; layouts, output
    dtypes and group sizes this build cannot honour exactly are refused; CPU
    tensors reach the wrappers' RuntimeError."""
    import torch

    from minixmax_h3_b200 import ops

    x = torch.randn(2, 3, 512)
    w = torch.zeros(64, 512, dtype=torch.int8)
    ws = torch.ones(64, dtype=torch.float64)
    with pytest.raises(RuntimeError):
        ops.int8_convrot_linear(x, w, ws)  # CPU tensors: no fallback
    with pytest.raises(ValueError):
        ops.int8_convrot_linear(x, w, ws, weight_layout="kn")
    with pytest.raises(NotImplementedError):
        ops.int8_convrot_linear(x, w, ws, out_dtype=torch.float16)
    with pytest.raises(NotImplementedError):
        ops.rotate_activation(x, 128)

    seen = {}

    def fake_quant(x2, *, convrot_group=0, x_rot_out=None):
        seen["quant"] = (x2.shape, x2.dtype, convrot_group)
        if x_rot_out is not None:
            x_rot_out.copy_(x2 * 2)
        return torch.zeros(x2.shape, dtype=torch.int8), torch.ones(x2.shape[0])

    def fake_gemm(q, xs, w_, ws_, b):
        seen["gemm"] = (q.shape, w_ is w, ws_.dtype, None if b is None else b.dtype)
        return torch.zeros(q.shape[0], w_.shape[0], dtype=torch.bfloat16)

    monkeypatch.setattr(ops, "quant_i8_rows", fake_quant)
    monkeypatch.setattr(ops, "gemm_i8", fake_gemm)
    y = ops.int8_convrot_linear(x, w, ws, torch.zeros(64))
    assert y.shape == (2, 3, 64) and y.dtype == torch.bfloat16
    assert seen["quant"] == ((6, 512), torch.bfloat16, 256)
    assert seen["gemm"] == ((6, 512), True, torch.float32, torch.bfloat16)
    ops.int8_convrot_linear(x, w, ws, convrot=False)
    assert seen["quant"][2] == 0
    xr = torch.randn(4, 512).to(torch.bfloat16)
    assert torch.equal(ops.rotate_activation(xr, 256), xr * 2)
