"""GPU parity of the drop-in modules and the fused DiT block.

References: the golden blocks were produced by the reference's own DiTBlock
(model/dit.py:400-438) with its projections evaluated by the oracle's
emulated quantised linear; the oracle block restates the same code path with
fp32 attention.  Bar: helpers.assert_close_bf16 (scaled max-abs <= 2e-2,
cosine >= 0.9995)."""
from __future__ import annotations

import pytest
import torch

from golden.make_golden import block_fixture_params
from helpers import assert_close_bf16, load_golden
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

FMT = {"int8": "int8_tensorwise", "nvfp4": "nvfp4"}


def _build_block(g, params, cuda):
    from minixmax_h3_b200.block import DiTBlock, load_quant_linear

    hidden = g["hidden"]
    blk = DiTBlock(hidden, g["heads"], 128, 4 * hidden, g["t_dim"], g["eps"], g["qk_eps"], apply_silu=True,
                   dtype=torch.bfloat16, device=cuda, mlp_act=g["mlp_act"])
    for mod, name in ((blk.attn.qkv_proj, "qkv"), (blk.attn.out_proj, "out"), (blk.mlp.fc1, "fc1"),
                      (blk.mlp.fc2, "fc2")):
        load_quant_linear(mod, params[f"{name}_w"].to(cuda), FMT[g["fmt"]])
    blk.norm1.weight.data.copy_(params["norm1_w"])
    blk.norm2.weight.data.copy_(params["norm2_w"])
    blk.attn.q_norm.weight.data.copy_(params["q_norm_w"])
    blk.attn.k_norm.weight.data.copy_(params["k_norm_w"])
    blk.adaln_proj.linear.weight.data.copy_(params["adaln_w"])
    blk.adaln_proj.linear.bias.data.copy_(params["adaln_b"])
    return blk


@pytest.mark.parametrize("name", ["dit_block_int8_gelu.pt", "dit_block_nvfp4_gelu.pt", "dit_block_nvfp4_swiglu.pt"])
def test_block_matches_reference_golden(cuda, name):
    from minixmax_h3_b200.block import RopeSpec

    g = load_golden(name)
    params = block_fixture_params(g)
    blk = _build_block(g, params, cuda)
    rope = RopeSpec(g["pos"].to(cuda), g["inv_freq"].to(cuda), g["n_t"], g["n_h"])
    x = g["x"].to(cuda).clone()
    out = blk(x, g["t_emb"].to(cuda), g["segments"], rope)
    assert out.data_ptr() == x.data_ptr()  # updated in place, like the reference
    assert_close_bf16(out, g["out"])
    lin = {n: O.EmulatedQuantLinear(params[f"{n}_w"], g["fmt"]) for n in ("qkv", "out", "fc1", "fc2")}
    want = O.dit_block_forward(g["x"].clone(), g["t_emb"], g["segments"], params, heads=g["heads"], head_dim=128,
                               eps=g["eps"], qk_eps=g["qk_eps"], mlp_act=g["mlp_act"], pos=g["pos"],
                               inv_freq=g["inv_freq"], n_t=g["n_t"], n_h=g["n_h"],
                               linear=lambda n, v: lin[n](v), attn_fp32=True)
    assert_close_bf16(out, want)
    # tokens outside every segment are neither modulated nor gated
    tail = slice(g["segments"][-1][1], None)
    assert_close_bf16(out[tail], g["out"][tail])


@pytest.mark.parametrize("fmt", ["int8_tensorwise", "nvfp4"])
def test_quant_linear_drop_in(cuda, fmt):
    """QuantLinear built from checkpoint tensors (from_quant_tensors, as the
    reference's loader does) matches the oracle's emulated linear, for 3D and
    fp32 inputs, with bias."""
    from minixmax_h3_b200.modules import QuantLinear

    gen = torch.Generator().manual_seed(2)
    n, k = 384, 512
    w = torch.randn(n, k, generator=gen) * 0.02
    bias = (0.1 * torch.randn(n, generator=gen)).to(torch.bfloat16)
    if fmt == "int8_tensorwise":
        wq, ws = O.quantize_weight_int8(w)
        ql = QuantLinear.from_quant_tensors(wq, meta={"format": fmt}, weight_scale=ws, bias=bias, device=cuda)
    else:
        qz = O.nvfp4_quantize(w.to(torch.bfloat16), hi_first=True)
        ql = QuantLinear.from_quant_tensors(qz["codes"], meta={"format": fmt},
                                            weight_scale=qz["sf"].view(torch.float8_e4m3fn),
                                            weight_scale_2=qz["gs"], bias=bias, device=cuda)
    ql.prepare_cube()
    x = torch.randn(2, 150, k, generator=gen)
    y = ql(x.to(cuda))  # fp32 input -> bf16 compute/output, as the reference
    assert y.shape == (2, 150, n) and y.dtype == torch.bfloat16
    emu = O.EmulatedQuantLinear(w if fmt == "int8_tensorwise" else w.to(torch.bfloat16),
                                "int8" if fmt == "int8_tensorwise" else "nvfp4", bias)
    assert_close_bf16(y, emu(x.to(torch.bfloat16)))
    with pytest.raises(RuntimeError):
        ql(x)  # CPU tensors: no fallback


def test_attention_entry_bnsd(cuda):
    from minixmax_h3_b200.attention import h3_attention_bnsd

    g = load_golden("attention.pt")
    out = h3_attention_bnsd(g["q"].to(cuda), g["k"].to(cuda), g["v"].to(cuda))
    assert out.shape == g["q"].shape
    assert_close_bf16(out, g["out"])


def test_dit_step_two_blocks(cuda):
    """condition_proj + 2 blocks over [text | video] vs the oracle chain."""
    from minixmax_h3_b200.block import DiTStep, RopeSpec, timestep_embedding

    hidden, heads, ffn, text_dim, n_text = 256, 2, 1024, 512, 16
    step = DiTStep(hidden=hidden, heads=heads, ffn=ffn, depth=2, text_dim=text_dim, fmt="nvfp4", mlp_act="gelu",
                   device=cuda)
    step.init_random(seed=3)
    gen = torch.Generator().manual_seed(5)
    grid = (2, 4, 8)
    pos = torch.cat([torch.stack([torch.arange(n_text, dtype=torch.float32), torch.zeros(n_text),
                                  torch.zeros(n_text)], -1), RopeSpec.grid_positions(*grid)])
    rope = RopeSpec.build(pos, device=cuda)
    video = torch.randn(pos.shape[0] - n_text, hidden, generator=gen).to(torch.bfloat16)
    text = torch.randn(n_text, text_dim, generator=gen).to(torch.bfloat16)
    ts = torch.tensor([437.0])
    out = step(video.to(cuda), text.to(cuda), ts.to(cuda), rope)

    # oracle: same quantised weights (read back from the modules), CPU math
    def lin_of(ql):
        codes = ql.weight_u8.cpu()
        qz = {"codes": codes, "sf": ql.weight_scale.cpu(), "gs": ql.weight_scale_2.cpu()}
        k = ql.in_features

        def f(v):
            a = O.nvfp4_quantize(v.reshape(-1, k).to(torch.bfloat16), hi_first=True)
            return O.nvfp4_linear_w4a4(a, qz, k).to(torch.bfloat16).reshape(*v.shape[:-1], -1)
        return f

    x = torch.cat([lin_of(step.condition_proj)(text), video])
    segs = [(0, n_text, 1), (n_text, pos.shape[0], 0)]
    t_emb = timestep_embedding(ts, 256).to(torch.bfloat16)
    for blk in step.blocks:
        p = {"adaln_w": blk.adaln_proj.linear.weight.cpu(), "adaln_b": blk.adaln_proj.linear.bias.cpu(),
             "norm1_w": blk.norm1.weight.cpu(), "norm2_w": blk.norm2.weight.cpu(),
             "q_norm_w": blk.attn.q_norm.weight.cpu(), "k_norm_w": blk.attn.k_norm.weight.cpu()}
        lins = {"qkv": lin_of(blk.attn.qkv_proj), "out": lin_of(blk.attn.out_proj), "fc1": lin_of(blk.mlp.fc1),
                "fc2": lin_of(blk.mlp.fc2)}
        x = O.dit_block_forward(x, t_emb, segs, p, heads=heads, head_dim=128, eps=1e-6, qk_eps=1e-6,
                                mlp_act="gelu", pos=pos, inv_freq=rope.inv_freq.cpu(), n_t=22, n_h=21,
                                linear=lambda n, v, lins=lins: lins[n](v), attn_fp32=True)
    assert_close_bf16(out, x)
