"""Regenerates the golden fixtures in this directory from the REFERENCE's own
Python (BHUHD/minixmax-h3, imported through oracle/reference.py).

    python tests/golden/make_golden.py

Each fixture stores seeded inputs and the reference's outputs for one hot-path
function, so the GPU tests can check the CUDA kernels against the reference on
machines where the reference tree is absent.  Fixtures:

  int8_quant.pt   ops/int8_convrot.py:99-111  _dynamic_quant_rows
  convrot.pt      ops/hadamard.py:35-44       rotate_activation (bf16 and fp16) + _dynamic_quant_rows
  nvfp4.pt        ops/nvfp4.py:124-151        dequantize_nvfp4 of oracle-quantised codes
  rope.pt         ops/rope.py:7-55            rope_rotation_table + rms_rope_apply (44/42/42)
  attention.pt    ops/attention.py:100-131    fusion_attention_bnsd (SDPA host path)
  dit_block_*.pt  model/dit.py:400-438        DiTBlock.forward with emulated quantised linears
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE.parent))

from oracle import h3_oracle as O  # noqa: E402
from oracle import reference  # noqa: E402

from golden.fixture_params import block_fixture_params  # noqa: E402,F401  (re-exported)


def outlier_activations(g: torch.Generator, m: int, k: int) -> torch.Tensor:
    """N(0,1) with 0.1% of entries scaled x20 (the benchmark's activation model)."""
    x = torch.randn(m, k, generator=g)
    mask = torch.rand(m, k, generator=g) < 0.001
    return torch.where(mask, x * 20.0, x)


def make_int8(R) -> dict:
    g = torch.Generator().manual_seed(0)
    x = outlier_activations(g, 46, 3072)
    x = torch.cat([x, torch.zeros(1, 3072), torch.full((1, 3072), 1e-30)], dim=0).to(torch.bfloat16)
    q, s = R.int8_convrot._dynamic_quant_rows(x.to(torch.bfloat16))
    return {"x": x, "q": q, "scale": s}


def make_convrot(R) -> dict:
    """The reference's online rotation (a 16-bit torch.mm against its regular
    Hadamard matrix) followed by its row quantiser, for bf16 and fp16 input."""
    g = torch.Generator().manual_seed(5)
    x = outlier_activations(g, 16, 3072)
    out = {}
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        xd = x.to(dt)
        rot = R.hadamard.rotate_activation(xd, 256)
        q, s = R.int8_convrot._dynamic_quant_rows(rot)
        out.update({f"x_{name}": xd, f"rot_{name}": rot, f"q_{name}": q, f"scale_{name}": s})
    return out


def make_nvfp4(R) -> dict:
    g = torch.Generator().manual_seed(1)
    x = outlier_activations(g, 130, 256)
    x[5] = 0.0
    x[7, 3] = 300.0
    x = x.to(torch.bfloat16)
    qz = O.nvfp4_quantize(x, hi_first=True)
    sf8 = qz["sf"].view(torch.float8_e4m3fn)
    deq = R.nvfp4.dequantize_nvfp4(qz["codes"], qz["gs"], sf8, out_dtype=torch.float32)
    deq_bf16 = R.nvfp4.dequantize_nvfp4(qz["codes"], qz["gs"], sf8, out_dtype=torch.bfloat16)
    return {"x": x, "codes_hi_first": qz["codes"], "sf": qz["sf"], "gs": qz["gs"], "dequant_f32": deq,
            "dequant_bf16": deq_bf16}


def make_rope(R) -> dict:
    g = torch.Generator().manual_seed(2)
    t, h, w = 2, 6, 8
    pos = O.grid_positions(t, h, w)
    heads = 3
    q = torch.randn(1, pos.shape[0], heads, 128, generator=g).to(torch.bfloat16) * 3
    weight = (1.0 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    inv = O.rope_inv_freq((44, 42, 42))
    angles = O.rope_angles(pos, inv, 22, 21)
    table = R.rope.rope_rotation_table(angles, torch.bfloat16)
    out = R.rope.rms_rope_apply(q, table, weight, 1e-6, 128)
    return {"q": q, "weight": weight, "pos": pos, "inv_freq": inv, "n_t": 22, "n_h": 21, "eps": 1e-6,
            "table": table, "out": out}


def make_attention(R) -> dict:
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 2, 200, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 2, 333, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 2, 333, 128, generator=g).to(torch.bfloat16)
    out = R.attention.fusion_attention_bnsd(q, k, v)
    return {"q": q, "k": k, "v": v, "out": out}


BLOCK_CFG = {"hidden": 256, "heads": 2, "t_dim": 32, "eps": 1e-6, "qk_eps": 1e-6, "grid": (1, 8, 16)}


def make_block(R, fmt: str, mlp_act: str, seed: int = 4) -> dict:
    """Reference DiTBlock with its four projections swapped for the oracle's
    emulated quantised linear (the only part the reference cannot run on CPU)."""
    c = BLOCK_CFG
    hidden, heads, t_dim, eps, qk_eps, grid = c["hidden"], c["heads"], c["t_dim"], c["eps"], c["qk_eps"], c["grid"]
    s_len = grid[0] * grid[1] * grid[2]
    ffn = 4 * hidden
    fix = {"seed": seed, "fmt": fmt, "mlp_act": mlp_act, "hidden": hidden, "heads": heads, "t_dim": t_dim,
           "eps": eps, "qk_eps": qk_eps, "grid": grid}
    p = block_fixture_params(fix)
    g = torch.Generator().manual_seed(seed + 1000)
    x = torch.randn(s_len, hidden, generator=g).to(torch.bfloat16)
    t = torch.rand(1, generator=g) * 1000.0
    t_emb = O.timestep_embedding(t, t_dim).to(torch.bfloat16)
    segments = [(0, s_len // 4, 1), (s_len // 4, s_len - 8, 0)]  # last 8 tokens: in no segment

    blk = R.dit.DiTBlock(hidden, heads, 128, ffn, t_dim, eps, qk_eps, apply_silu=True, dtype=torch.bfloat16)
    blk.norm1.weight.data.copy_(p["norm1_w"])
    blk.norm2.weight.data.copy_(p["norm2_w"])
    blk.attn.q_norm.weight.data.copy_(p["q_norm_w"])
    blk.attn.k_norm.weight.data.copy_(p["k_norm_w"])
    blk.adaln_proj.linear.weight.data.copy_(p["adaln_w"])
    blk.adaln_proj.linear.bias.data.copy_(p["adaln_b"])
    lin = {n: O.EmulatedQuantLinear(p[f"{n}_w"], fmt) for n in ("qkv", "out", "fc1", "fc2")}
    blk.attn.qkv_proj = lin["qkv"]
    blk.attn.out_proj = lin["out"]
    blk.mlp.fc1 = lin["fc1"]
    blk.mlp.fc2 = lin["fc2"]
    if mlp_act == "gelu":
        blk.mlp.forward = lambda u: lin["fc2"](F.gelu(lin["fc1"](u)))

    pos = O.grid_positions(*grid)
    inv = O.rope_inv_freq((44, 42, 42))
    table = R.rope.rope_rotation_table(O.rope_angles(pos, inv, 22, 21), torch.bfloat16)
    with torch.no_grad():
        out = blk(x.clone(), t_emb, segments, table)
    fix.update({"segments": segments, "x": x, "t_emb": t_emb, "pos": pos, "inv_freq": inv, "n_t": 22, "n_h": 21,
                "out": out})
    return fix


def main() -> None:
    R = reference.load()
    if R is None:
        raise SystemExit("reference tree not found; set H3B_REFERENCE_ROOT")
    torch.set_num_threads(1)
    fixtures = {
        "int8_quant.pt": make_int8(R),
        "convrot.pt": make_convrot(R),
        "nvfp4.pt": make_nvfp4(R),
        "rope.pt": make_rope(R),
        "attention.pt": make_attention(R),
        "dit_block_int8_gelu.pt": make_block(R, "int8", "gelu"),
        "dit_block_nvfp4_gelu.pt": make_block(R, "nvfp4", "gelu"),
        "dit_block_nvfp4_swiglu.pt": make_block(R, "nvfp4", "swiglu"),
    }
    for name, data in fixtures.items():
        torch.save(data, HERE / name)
        print(f"wrote {name} ({(HERE / name).stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
