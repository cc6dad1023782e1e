"""GPU parity at BASELINE's own shapes.

cfg 1: one DiT block, hidden 1024, 8 heads x 128, 4096 tokens on the latent
grid t4 x h32 x w32, INT8 W8A8 (per-channel weight scales, per-token dynamic
activation scales), GELU MLP 4x, adaLN from a 256-d sinusoidal timestep
embedding, seed 0 — against the oracle's block (model/dit.py:400-438 restated,
pinned bit-exact to the reference's DiTBlock by tests/test_oracle_pins.py),
plus the INT8 activation codes and int32 accumulators of its QKV projection,
bit-exact.

cfg 5 (sampled): one block of the benchmarked stack — hidden 3072, 24 heads,
GELU MLP 12288, NVFP4 W4A4 — over the full S = 498,272 tokens (512 text rows
on adaLN row 1, then video rows).  The GPU runs every stage over all tokens;
the CPU re-derives sampled rows of each stage from the GPU's own input to
that stage: the norm + modulate rows, the activation codes and block scales
(bit-exact, with the whole tensor's global scale), the QKV GEMM rows, the
q/k RMSNorm + RoPE rows, the attention rows of two heads (including the last
rows and the partial last K/V tile: 498,272 mod 128 = 96) against all keys,
the out-projection with its gate-residual epilogue, fc1 (bf16 output and
its max), the GELU applied inside fc2's input quantiser (codes and scales
bit-exact against the oracle's quantisation of F.gelu of fc1's output, with
max |u| from max y checked against the full maximum) and fc2 with its
gate-residual epilogue.  Bars: bit-exact for codes, scales and
accumulators; helpers.assert_close_bf16 (scaled max-abs <= 2e-2, cosine >=
0.9995) for bf16 outputs, 1e-2 for the norm and RoPE rows as in their own
tests.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close_bf16
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu


def _block(cuda, hidden, heads, fmt, gen, mlp_act="gelu"):
    from minixmax_h3_b200.block import DiTBlock, load_quant_linear

    blk = DiTBlock(hidden, heads, 128, 4 * hidden, 256, 1e-6, 1e-6, apply_silu=True, dtype=torch.bfloat16,
                   device=cuda, mlp_act=mlp_act)
    inner = heads * 128
    w = {"qkv": torch.randn(3 * inner, hidden, generator=gen) * 0.02,
         "out": torch.randn(hidden, inner, generator=gen) * 0.02,
         "fc1": torch.randn(4 * hidden, hidden, generator=gen) * 0.02,
         "fc2": torch.randn(hidden, 4 * hidden, generator=gen) * 0.02}
    for name, mod in (("qkv", blk.attn.qkv_proj), ("out", blk.attn.out_proj), ("fc1", blk.mlp.fc1),
                      ("fc2", blk.mlp.fc2)):
        load_quant_linear(mod, w[name].to(cuda), fmt)
    p = {"adaln_w": (torch.randn(6 * hidden * 3, 256, generator=gen) * 0.02).to(torch.bfloat16),
         "adaln_b": (torch.randn(6 * hidden * 3, generator=gen) * 0.02).to(torch.bfloat16)}
    for name in ("norm1_w", "norm2_w"):
        p[name] = (1.0 + 0.1 * torch.randn(hidden, generator=gen)).to(torch.bfloat16)
    for name in ("q_norm_w", "k_norm_w"):
        p[name] = (1.0 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    blk.adaln_proj.linear.weight.data.copy_(p["adaln_w"])
    blk.adaln_proj.linear.bias.data.copy_(p["adaln_b"])
    blk.norm1.weight.data.copy_(p["norm1_w"])
    blk.norm2.weight.data.copy_(p["norm2_w"])
    blk.attn.q_norm.weight.data.copy_(p["q_norm_w"])
    blk.attn.k_norm.weight.data.copy_(p["k_norm_w"])
    return blk, w, p


def test_cfg1_block_int8_gelu(cuda):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.block import RopeSpec, timestep_embedding

    hidden, heads, grid = 1024, 8, (4, 32, 32)
    gen = torch.Generator().manual_seed(0)
    blk, w, p = _block(cuda, hidden, heads, "int8_tensorwise", gen)
    pos = RopeSpec.grid_positions(*grid)
    s_len = pos.shape[0]
    assert s_len == 4096
    rope = RopeSpec.build(pos, device=cuda)
    x = torch.randn(s_len, hidden, generator=gen).to(torch.bfloat16)  # fp32 N(0,1), cast as the reference does
    t = torch.rand(1, generator=gen) * 1000.0
    t_emb = timestep_embedding(t, 256).to(torch.bfloat16)
    segs = [(0, s_len, 0)]

    # stage: norm1 + modulate (float bar: the fp32 sum of squares is reduced
    # in another order on the CPU, so h can differ by a bf16 ulp), then the
    # per-token INT8 codes of the QKV input from the GPU's own h and the QKV
    # int32 accumulators, bit-exact
    shift, scale, *_ = blk.adaln_proj(t_emb.to(cuda))
    sel = torch.zeros(s_len, dtype=torch.int32, device=cuda)
    h = ops.rmsnorm_modulate(x.to(cuda), blk.norm1.weight, shift, scale, 1e-6, row_sel=sel)
    h_ref = O.mod_scale_shift(O.rms_norm(x, p["norm1_w"], 1e-6), shift.cpu(), scale.cpu(), segs)
    assert_close_bf16(h, h_ref, max_abs=1e-2)
    q, xs = ops.rmsnorm_modulate_quant_i8(x.to(cuda), blk.norm1.weight, shift, scale, 1e-6, row_sel=sel)
    q_ref, xs_ref = O.dynamic_quant_rows(h.cpu())
    assert torch.equal(q.cpu(), q_ref) and torch.equal(xs.cpu(), xs_ref)
    rows = torch.randperm(s_len, generator=gen)[:256]
    acc = ops.gemm_i8_acc(q, blk.attn.qkv_proj.weight_i8)
    assert torch.equal(acc.cpu()[rows], O.int8_acc(q_ref[rows], blk.attn.qkv_proj.weight_i8.cpu()))

    out = blk(x.to(cuda), t_emb.to(cuda), segs, rope)
    lin = {n: O.EmulatedQuantLinear(w[n], "int8") for n in w}
    want = O.dit_block_forward(x.clone(), t_emb, segs, p, heads=heads, head_dim=128, eps=1e-6, qk_eps=1e-6,
                               mlp_act="gelu", pos=pos, inv_freq=rope.inv_freq.cpu(), n_t=rope.n_t, n_h=rope.n_h,
                               linear=lambda n, v: lin[n](v), attn_fp32=True)
    assert_close_bf16(out, want)


# ----------------------------------------------------------------------------- cfg 5, sampled


def _take(t: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """Rows of a (large) device tensor, gathered on the device, then copied."""
    return t[rows.to(t.device)].cpu()


def _nvfp4_rows(t, rows: torch.Tensor, k: int) -> dict:
    """Codes (hi-first, as the oracle packs them), blocked scales and gs of
    the sampled rows of a GPU NVFP4Tensor (lo-first codes)."""
    codes = O.swap_nibbles(_take(t.codes, rows))
    ncols = k // 16
    r = rows.numpy()[:, None]
    c = np.arange(ncols)[None, :]
    offs = torch.from_numpy(O.blocked_offset(r, c, ncols).astype(np.int64))
    dense = t.sf[offs.reshape(-1).to(t.sf.device)].cpu().reshape(rows.numel(), ncols).numpy()
    return {"codes": codes, "sf_logical": torch.from_numpy(np.ascontiguousarray(dense)),
            "sf": torch.from_numpy(O.to_blocked(np.ascontiguousarray(dense))), "gs": t.gs.cpu()}


def _check_quant(t, x_gpu, rows, k, amax: torch.Tensor):
    """GPU codes / scales of the sampled rows == the oracle's quantisation of
    the same rows with the whole tensor's global scale (from its |max|)."""
    got = _nvfp4_rows(t, rows, k)
    want = O.nvfp4_quantize(_take(x_gpu, rows), hi_first=True, amax=amax.item())
    assert torch.equal(got["gs"], want["gs"])
    assert torch.equal(got["codes"], want["codes"])
    assert torch.equal(got["sf_logical"], want["sf_logical"])
    return got


def _w_dict(ql) -> dict:
    return {"codes": ql.weight_u8.cpu(), "sf": ql.weight_scale.cpu(), "gs": ql.weight_scale_2.cpu()}


def test_cfg5_block_sampled_stages(cuda):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.block import RopeSpec, init_block_random, timestep_embedding
    from minixmax_h3_b200.ops import EPI_GATE_RES, EPI_STORE_POSMAX

    hidden, heads, n_text, grid = 3072, 24, 512, (61, 68, 120)
    ffn = 4 * hidden
    text_pos = torch.stack([torch.arange(n_text, dtype=torch.float32), torch.zeros(n_text), torch.zeros(n_text)], -1)
    pos = torch.cat([text_pos, RopeSpec.grid_positions(*grid)])
    s_len = pos.shape[0]
    assert s_len == 498272 and s_len % 128 == 96
    rope = RopeSpec.build(pos, device=cuda)
    from minixmax_h3_b200.block import DiTBlock

    blk = DiTBlock(hidden, heads, 128, ffn, 256, 1e-6, 1e-6, apply_silu=True, dtype=torch.bfloat16, device=cuda,
                   mlp_act="gelu")
    init_block_random(blk, "nvfp4", torch.Generator(device=cuda).manual_seed(0))
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(s_len, hidden, generator=g, device=cuda).to(torch.bfloat16)
    t_emb = timestep_embedding(torch.tensor([500.0], device=cuda), 256).to(torch.bfloat16)
    shift1, scale1, gate1, shift2, scale2, gate2 = blk.adaln_proj(t_emb)
    sel = torch.cat([torch.ones(n_text, dtype=torch.int32), torch.zeros(s_len - n_text, dtype=torch.int32)]
                    ).to(cuda)
    cg = torch.Generator().manual_seed(2)
    # sampled rows: text rows first (adaLN row 1), then video rows (row 0),
    # including the sequence's last rows
    text_rows = torch.randperm(n_text, generator=cg)[:32].sort().values
    video_rows = (n_text + torch.randperm(s_len - n_text - 64, generator=cg)[:96]).sort().values
    rows = torch.cat([text_rows, video_rows, torch.arange(s_len - 64, s_len)])
    segs = [(0, 32, 1), (32, rows.numel(), 0)]  # of the sampled rows, in their order
    cpu = {n: t.cpu() for n, t in (("shift1", shift1), ("scale1", scale1), ("gate1", gate1), ("shift2", shift2),
                                   ("scale2", scale2), ("gate2", gate2))}

    # norm1 + modulate (+ global |h| max)
    amax_h = torch.zeros(1, dtype=torch.float32, device=cuda)
    h = ops.rmsnorm_modulate(x, blk.norm1.weight, shift1, scale1, 1e-6, row_sel=sel, amax_out=amax_h)
    h_ref = O.mod_scale_shift(O.rms_norm(_take(x, rows), blk.norm1.weight.cpu(), 1e-6), cpu["shift1"],
                              cpu["scale1"], segs)
    assert_close_bf16(_take(h, rows), h_ref, max_abs=1e-2)
    assert amax_h.item() == h.abs().max().float().item()

    # activation quantisation + QKV GEMM
    ql = blk.attn.qkv_proj
    ql.prepare_cube()
    a = ops.quant_nvfp4(h, amax_t=amax_h)
    a_rows = _check_quant(a, h, rows, hidden, amax_h)
    qkv = ops.gemm_nvfp4(a, ql._w_nvfp4)
    assert_close_bf16(_take(qkv, rows), O.nvfp4_linear_w4a4(a_rows, _w_dict(ql), hidden))

    # q/k RMSNorm + RoPE, in place over the packed QKV output
    q3 = qkv.view(s_len, 3, heads, 128)
    pre = _take(q3, rows)
    ops.qk_rmsnorm_rope(q3[:, 0], q3[:, 1], blk.attn.q_norm.weight, blk.attn.k_norm.weight, 1e-6, rope.pos, 0,
                        rope.inv_freq, rope.n_t, rope.n_h)
    table = O.rope_rotation_table(O.rope_angles(pos[rows], rope.inv_freq.cpu(), rope.n_t, rope.n_h),
                                  torch.bfloat16)
    for part, wname in ((0, "q_norm"), (1, "k_norm")):
        want = O.rms_rope_apply(pre[:, part].unsqueeze(0).clone(), table, getattr(blk.attn, wname).weight.cpu(),
                                1e-6, 128)[0]
        assert_close_bf16(_take(q3, rows)[:, part], want, max_abs=1e-2)

    # attention over all keys (two heads checked: rows incl. the last 64, so
    # the partial last K/V tile is in every row's softmax)
    amax_o = torch.zeros(1, dtype=torch.float32, device=cuda)
    o = ops.attention(q3[:, 0], q3[:, 1], q3[:, 2], amax_out=amax_o)
    for hd in (0, heads - 1):
        qh = _take(q3[:, 0, hd], rows).float()
        kh, vh = q3[:, 1, hd].cpu().float(), q3[:, 2, hd].cpu().float()
        p_ = torch.softmax((qh @ kh.T) * 128 ** -0.5, dim=-1)
        assert_close_bf16(_take(o[:, hd], rows), (p_ @ vh).to(torch.bfloat16))
        del p_, kh, vh
    assert amax_o.item() == o.abs().max().float().item()

    # out-projection with the gate-residual epilogue: x += gate1 * out(o)
    x_before = _take(x, rows)
    qo = blk.attn.out_proj
    qo.prepare_cube()
    ao = ops.quant_nvfp4(o.view(s_len, hidden), amax_t=amax_o)
    ao_rows = _check_quant(ao, o.view(s_len, hidden), rows, hidden, amax_o)
    ops.gemm_nvfp4(ao, qo._w_nvfp4, epilogue=EPI_GATE_RES, resid=x, gate=gate1, row_sel=sel)
    y_ref = O.nvfp4_linear_w4a4(ao_rows, _w_dict(qo), hidden).to(torch.bfloat16)
    assert_close_bf16(_take(x, rows), O.mod_gate(x_before.clone(), cpu["gate1"], y_ref, segs))

    # norm2 + modulate, fc1 storing its bf16 output y and max(0, max y)
    amax_h2 = torch.zeros(1, dtype=torch.float32, device=cuda)
    h2 = ops.rmsnorm_modulate(x, blk.norm2.weight, shift2, scale2, 1e-6, row_sel=sel, amax_out=amax_h2)
    f1 = blk.mlp.fc1
    f1.prepare_cube()
    a2 = ops.quant_nvfp4(h2, amax_t=amax_h2)
    a2_rows = _check_quant(a2, h2, rows, hidden, amax_h2)
    ymax2 = torch.zeros(2, dtype=torch.float32, device=cuda)
    y = ops.gemm_nvfp4(a2, f1._w_nvfp4, epilogue=EPI_STORE_POSMAX, amax_out=ymax2[:1])
    y_ref = O.nvfp4_linear_w4a4(a2_rows, _w_dict(f1), hidden).to(torch.bfloat16)
    assert_close_bf16(_take(y, rows), y_ref)
    assert ymax2[0].item() == max(0.0, y.max().float().item())

    # GELU inside fc2's input quantiser: u = bf16(gelu(y)) (torch's F.gelu of
    # the bf16 output on the GPU is the same chain); max |u| from max y
    ops.gelu_amax_scan(y, ymax2)
    assert ymax2[1].item() == 0.0  # the bound settles max |u| at this scale
    amax_u = F.gelu(ymax2[:1].to(torch.bfloat16)).float()
    chunk = 1 << 16
    assert max(F.gelu(y[i:i + chunk]).abs().max().float().item() for i in range(0, s_len, chunk)) == amax_u.item()
    au = ops.quant_nvfp4_gelu(y, ymax2)
    au_rows = _nvfp4_rows(au, rows, ffn)
    want = O.nvfp4_quantize(F.gelu(y[rows.to(cuda)]).cpu(), hi_first=True, amax=amax_u.item())
    assert torch.equal(au_rows["gs"], want["gs"])
    assert torch.equal(au_rows["codes"], want["codes"])
    assert torch.equal(au_rows["sf_logical"], want["sf_logical"])

    # fc2 with the gate-residual epilogue
    x_before = _take(x, rows)
    f2 = blk.mlp.fc2
    f2.prepare_cube()
    ops.gemm_nvfp4(au, f2._w_nvfp4, epilogue=EPI_GATE_RES, resid=x, gate=gate2, row_sel=sel)
    y2 = O.nvfp4_linear_w4a4(au_rows, _w_dict(f2), ffn).to(torch.bfloat16)
    assert_close_bf16(_take(x, rows), O.mod_gate(x_before.clone(), cpu["gate2"], y2, segs))
