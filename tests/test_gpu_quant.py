"""GPU parity: activation quantisers vs the oracle and the reference fixtures.

Bar: INT8 codes/scales and NVFP4 codes/scales are bit-exact."""
from __future__ import annotations

import pytest
import torch

from helpers import load_golden
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu


def _outliers(seed: int, m: int, k: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    return torch.where(torch.rand(m, k, generator=g) < 0.001, 20 * x, x).to(torch.bfloat16)


def test_int8_golden(cuda):
    from minixmax_h3_b200 import ops

    g = load_golden("int8_quant.pt")
    q, s = ops.quant_i8_rows(g["x"].to(cuda))
    assert torch.equal(q.cpu(), g["q"]) and torch.equal(s.cpu(), g["scale"])


@pytest.mark.parametrize("k", [8, 72, 3072, 12288, 40960])
def test_int8_rows_bit_exact(cuda, k):
    from minixmax_h3_b200 import ops

    x = _outliers(k, 129, k)
    q, s = ops.quant_i8_rows(x.to(cuda))
    q_ref, s_ref = O.dynamic_quant_rows(x)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)


def test_int8_fp16_and_strided(cuda):
    from minixmax_h3_b200 import ops

    x = _outliers(3, 64, 1024).to(torch.float16)
    q, s = ops.quant_i8_rows(x.to(cuda))
    q_ref, s_ref = O.dynamic_quant_rows(x)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)
    big = _outliers(4, 64, 2048).to(cuda)
    q2, s2 = ops.quant_i8_rows(big[:, 512:1536])  # row stride 2048
    q2_ref, s2_ref = O.dynamic_quant_rows(big[:, 512:1536].cpu())
    assert torch.equal(q2.cpu(), q2_ref) and torch.equal(s2.cpu(), s2_ref)


def test_int8_cfg2_full_size_sampled(cuda):
    """M=32768 x K=12288 on the GPU; 512 random rows re-derived on the CPU."""
    from minixmax_h3_b200 import ops

    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(32768, 12288, generator=g, device=cuda)
    x = torch.where(torch.rand(32768, 12288, generator=g, device=cuda) < 0.001, 20 * x, x).to(torch.bfloat16)
    q, s = ops.quant_i8_rows(x)
    rows = torch.randperm(32768, generator=torch.Generator().manual_seed(1))[:512]
    q_ref, s_ref = O.dynamic_quant_rows(x[rows.to(cuda)].cpu())
    assert torch.equal(q[rows.to(cuda)].cpu(), q_ref) and torch.equal(s[rows.to(cuda)].cpu(), s_ref)


def test_nvfp4_golden(cuda):
    from minixmax_h3_b200 import ops

    g = load_golden("nvfp4.pt")
    hi = ops.quant_nvfp4(g["x"].to(cuda), hi_first=True)
    assert torch.equal(hi.codes.cpu(), g["codes_hi_first"])
    assert torch.equal(hi.sf.cpu(), g["sf"]) and torch.equal(hi.gs.cpu(), g["gs"])
    lo = ops.quant_nvfp4(g["x"].to(cuda), hi_first=False)
    assert torch.equal(O.swap_nibbles(lo.codes.cpu()), g["codes_hi_first"])
    assert torch.equal(ops.swap_nibbles(lo.codes).cpu(), g["codes_hi_first"])


@pytest.mark.parametrize("m,k", [(1, 64), (300, 3072), (4096, 3072), (257, 12288)])
def test_nvfp4_bit_exact(cuda, m, k):
    from minixmax_h3_b200 import ops

    x = _outliers(m + k, m, k)
    got = ops.quant_nvfp4(x.to(cuda), hi_first=True)
    want = O.nvfp4_quantize(x, hi_first=True)
    assert torch.equal(got.gs.cpu(), want["gs"])
    assert torch.equal(got.codes.cpu(), want["codes"])
    assert torch.equal(got.sf.cpu(), want["sf"])


@pytest.mark.parametrize("scale", [1.0, 1e-30, 1e25])
@pytest.mark.parametrize("hi_first", [True, False])
def test_nvfp4_wide_range_bit_exact(cuda, scale, hi_first):
    """Magnitudes spread over 2^-40 .. 2^40 within the tensor (blocks far
    below the global max, signed zeros, exact ties), at three overall
    scales, so the reciprocal-based division, its range guards and the
    exact-division fallback are all exercised."""
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(int(abs(torch.tensor(scale).log10())) + hi_first)
    m, k = 512, 1024
    mant = 1.0 + torch.rand(m, k, generator=g)
    expo = torch.randint(-40, 41, (m, k), generator=g).float()
    sign = torch.where(torch.rand(m, k, generator=g) < 0.5, -1.0, 1.0)
    x = sign * mant * torch.exp2(expo) * scale
    x[3] = 0.0
    x[4] = -0.0
    x[5, :64] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 8) * scale  # e2m1 ties
    x = x.to(torch.bfloat16)
    got = ops.quant_nvfp4(x.to(cuda), hi_first=hi_first)
    want = O.nvfp4_quantize(x, hi_first=hi_first)
    assert torch.equal(got.gs.cpu(), want["gs"])
    assert torch.equal(got.sf.cpu(), want["sf"])
    assert torch.equal(got.codes.cpu(), want["codes"])


def test_amax_and_zero_input(cuda):
    from minixmax_h3_b200 import ops

    x = _outliers(9, 333, 256)
    assert ops.amax(x.to(cuda)).item() == x.float().abs().max().item()
    z = torch.zeros(130, 128, dtype=torch.bfloat16)
    got = ops.quant_nvfp4(z.to(cuda), hi_first=True)
    want = O.nvfp4_quantize(z, hi_first=True)
    assert got.gs.item() == 1.0 and torch.equal(got.codes.cpu(), want["codes"]) and torch.equal(got.sf.cpu(), want["sf"])


# ---------------------------------------------------------------- ConvRot

def test_convrot_golden(cuda):
    """Rotated activation and codes vs the reference's rotate_activation +
    _dynamic_quant_rows: bit-exact for bf16; fp16 rotations within the
    reference GEMM's own 2-ulp rounding (the oracle pins that)."""
    from minixmax_h3_b200 import ops

    g = load_golden("convrot.pt")
    x = g["x_bf16"]
    rot = torch.empty_like(x, device=cuda)
    q, s = ops.quant_i8_rows(x.to(cuda), convrot_group=256, x_rot_out=rot)
    assert torch.equal(rot.cpu(), g["rot_bf16"])
    assert torch.equal(q.cpu(), g["q_bf16"]) and torch.equal(s.cpu(), g["scale_bf16"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k", [(1, 256), (37, 3072), (130, 4096), (64, 12288)])
def test_convrot_bit_exact(cuda, dtype, m, k):
    from minixmax_h3_b200 import ops

    x = _outliers(m + k, m, k).to(dtype)
    rot = torch.empty(m, k, dtype=dtype, device=cuda)
    q, s = ops.quant_i8_rows(x.to(cuda), convrot_group=256, x_rot_out=rot)
    rot_ref = O.rotate_activation_exact(x, 256)
    q_ref, s_ref = O.dynamic_quant_rows(rot_ref)
    assert torch.equal(rot.cpu(), rot_ref)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)


def test_convrot_strided_rows_and_zero(cuda):
    from minixmax_h3_b200 import ops

    base = _outliers(5, 20, 3072 + 64)
    base[3] = 0
    x = base[:, :3072]  # row pitch 3136 elements
    q, s = ops.quant_i8_rows(x.to(cuda), convrot_group=256)
    q_ref, s_ref = O.dynamic_quant_rows(O.rotate_activation_exact(x.contiguous(), 256))
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)
    assert (q[3] == 0).all()


def test_convrot_quantlinear(cuda):
    """QuantLinear with meta convrot: rotated W8A8 output bit-exact to the
    oracle's emulated linear (rotation, row quantisation, int32 product,
    fp32 epilogue, one bf16 rounding)."""
    from minixmax_h3_b200.modules import QuantLinear

    g = torch.Generator().manual_seed(3)
    x = _outliers(8, 200, 3072)
    w = torch.randn(512, 3072, generator=g) * 0.02
    emu = O.EmulatedQuantLinear(w, "int8", convrot=True)
    ql = QuantLinear.from_quant_tensors(emu.wq, meta={"format": "int8_tensorwise", "convrot": True},
                                        weight_scale=emu.ws, device=cuda)
    y = ql(x.to(cuda))
    assert torch.equal(y.cpu(), emu(x))


# ------------------------------------------------- fused norm + modulate + INT8

@pytest.mark.parametrize("hidden", [512, 3072, 12288])
@pytest.mark.parametrize("group", [0, 256])
def test_rmsnorm_modulate_quant_i8_matches_two_kernels(cuda, hidden, group):
    """One kernel == rmsnorm_modulate then quant_i8_rows(_convrot), bit for
    bit, including rows outside every modulation segment (row_sel -1)."""
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(hidden + group)
    m = 300
    x = (torch.randn(m, hidden, generator=g) * 3).to(torch.bfloat16).to(cuda)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16).to(cuda)
    tab = (0.2 * torch.randn(3, 2 * hidden, generator=g)).to(torch.bfloat16).to(cuda)
    shift, scale = tab[:, :hidden], tab[:, hidden:]
    sel = torch.randint(-1, 3, (m,), generator=g, dtype=torch.int32).to(cuda)
    q, xs = ops.rmsnorm_modulate_quant_i8(x, w, shift, scale, 1e-6, row_sel=sel, convrot_group=group)
    h = ops.rmsnorm_modulate(x, w, shift, scale, 1e-6, row_sel=sel)
    q_ref, xs_ref = ops.quant_i8_rows(h, convrot_group=group)
    assert torch.equal(q, q_ref) and torch.equal(xs, xs_ref)
    # and against the oracle's restatement of the same chain
    rot = O.rotate_activation_exact(h.cpu(), 256) if group else h.cpu()
    q_o, xs_o = O.dynamic_quant_rows(rot)
    assert torch.equal(q.cpu(), q_o) and torch.equal(xs.cpu(), xs_o)
