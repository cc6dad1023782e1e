"""GPU parity: tcgen05 INT8 and NVFP4 GEMMs.

Bars: int32 accumulators bit-exact; INT8 bf16 outputs bit-exact to the
oracle's fp32 epilogue ((acc*xs)*ws + bias, one bf16 rounding); NVFP4 and
activation epilogues within helpers.assert_close_bf16 (scaled max-abs <= 2e-2,
cosine >= 0.9995) of the exact fp64 product of the decoded operands."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close_bf16
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 128), (300, 288, 384), (1000, 3072, 3072), (64, 512, 12288)]


def _i8(seed, *shape):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_i8_acc_bit_exact(cuda, m, n, k):
    from minixmax_h3_b200 import ops

    q, w = _i8(m, m, k), _i8(n, n, k)
    acc = ops.gemm_i8_acc(q.to(cuda), w.to(cuda))
    assert torch.equal(acc.cpu(), O.int8_acc(q, w))


@pytest.mark.parametrize("m,n,k", SHAPES[:3])
def test_i8_linear_bit_exact(cuda, m, n, k):
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(7)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w, ws = O.quantize_weight_int8(torch.randn(n, k, generator=g) * 0.02)
    bias = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    q, xs = ops.quant_i8_rows(x.to(cuda))
    y = ops.gemm_i8(q, xs, w.to(cuda), ws.to(cuda), bias.to(cuda))
    q_ref, xs_ref = O.dynamic_quant_rows(x)
    assert torch.equal(q.cpu(), q_ref)
    assert torch.equal(y.cpu(), O.w8a8_linear(q_ref, xs_ref, w, ws, bias))


def test_i8_cfg2_shapes_sampled(cuda):
    """BASELINE cfg 2 shapes at full M; 256 random rows checked bit-exact."""
    from minixmax_h3_b200 import ops

    rows = torch.randperm(32768, generator=torch.Generator().manual_seed(2))[:256]
    for k, n in [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072)]:
        q = torch.randint(-128, 128, (32768, k), dtype=torch.int8, device=cuda)
        w = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=cuda)
        acc = ops.gemm_i8_acc(q, w)
        r = rows.to(cuda)
        assert torch.equal(acc[r].cpu(), O.int8_acc(q[r].cpu(), w.cpu())), (k, n)


def test_i8_epilogues(cuda):
    from minixmax_h3_b200 import ops

    m, n, k = 256, 512, 1024
    g = torch.Generator().manual_seed(9)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w, ws = O.quantize_weight_int8(torch.randn(n, k, generator=g) * 0.02)
    resid = torch.randn(m, n, generator=g).to(torch.bfloat16)
    gate = torch.randn(n, generator=g).to(torch.bfloat16)
    q, xs = ops.quant_i8_rows(x.to(cuda))
    y_lin = O.w8a8_linear(*O.dynamic_quant_rows(x), w, ws).float()
    pre = O.int8_acc(*[O.dynamic_quant_rows(x)[0], w]).float() * O.dynamic_quant_rows(x)[1][:, None] * ws[None]
    gelu = ops.gemm_i8(q, xs, w.to(cuda), ws.to(cuda), epilogue=ops.EPI_GELU)
    assert_close_bf16(gelu, F.gelu(pre), max_abs=1e-2)
    r = resid.to(cuda).clone()
    out = ops.gemm_i8(q, xs, w.to(cuda), ws.to(cuda), epilogue=ops.EPI_GATE_RES, resid=r, gate=gate.to(cuda))
    assert out.data_ptr() == r.data_ptr()
    want = (resid.float() + pre * gate.float()).to(torch.bfloat16)
    assert torch.equal(out.cpu(), want)
    assert_close_bf16(y_lin, pre)


def _nvfp4_operands(cuda, m, n, k, seed):
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x = torch.where(torch.rand(m, k, generator=g) < 0.001, 20 * x, x).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    a = ops.quant_nvfp4(x.to(cuda))
    wq = ops.quant_nvfp4(w.to(cuda))
    return x, w, a, wq


# n = 160 and 448 end in a partial 192-wide tile; 384 and 3072 exercise the odd
# tiles whose weight scales start 64 rows into a 128-row block.
@pytest.mark.parametrize(
    "m,n,k",
    [(128, 256, 256), (300, 384, 512), (1000, 3072, 3072), (200, 256, 12288), (64, 160, 512), (130, 448, 256)],
)
def test_nvfp4_gemm(cuda, m, n, k):
    from minixmax_h3_b200 import ops

    x, w, a, wq = _nvfp4_operands(cuda, m, n, k, m + n + k)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(1)) * 0.1).to(torch.bfloat16)
    y = ops.gemm_nvfp4(a, wq, bias.to(cuda))
    a_or = {"codes": a.codes.cpu(), "sf": a.sf.cpu(), "gs": a.gs.cpu()}
    w_or = {"codes": wq.codes.cpu(), "sf": wq.sf.cpu(), "gs": wq.gs.cpu()}
    exact = O.nvfp4_linear_w4a4(a_or, w_or, k, bias, a_hi_first=False, w_hi_first=False)
    assert_close_bf16(y, exact)
    # The reference's own arithmetic on the same codes (ops/nvfp4.py:154-173):
    # decode to bf16, then F.linear.  Rounding every decoded operand to bf16
    # (relative 2^-9 each) makes that path itself drift from the exact
    # product as sqrt(K) grows, so this comparison allows 5e-2 (scaled).
    ad = O.nvfp4_dequantize(a_or["codes"], a_or["gs"], a_or["sf"], k, False).to(torch.bfloat16)
    wd = O.nvfp4_dequantize(w_or["codes"], w_or["gs"], w_or["sf"], k, False).to(torch.bfloat16)
    assert_close_bf16(y, F.linear(ad, wd, bias).float(), max_abs=5e-2)


def test_nvfp4_cfg3_shapes_sampled(cuda):
    """BASELINE cfg 3 shapes at full M=32768: the whole activation and weight
    quantised on the GPU, then two 128-row groups of each (group 0 holds the
    planted global max, so a CPU quantiser of just those rows sees the same
    global scale) checked bit-exact in codes and blocked scales, and the
    GEMM's outputs at those rows and columns held to the float bar against
    the exact product of the decoded operands."""
    from minixmax_h3_b200 import ops

    m = 32768
    gen = torch.Generator().manual_seed(3)

    def sample(count):
        groups = [0, int(torch.randint(1, count // 128, (1,), generator=gen))]
        return groups, torch.cat([torch.arange(g * 128, g * 128 + 128) for g in groups])

    def check_rows(t, src, groups, rows, k):
        ref = O.nvfp4_quantize(src[rows.to(cuda)].cpu(), hi_first=False)
        chunk = (k // 16 + 3) // 4 * 512  # blocked scale bytes of one 128-row group
        assert torch.equal(t.gs.cpu(), ref["gs"])
        assert torch.equal(t.codes[rows.to(cuda)].cpu(), ref["codes"])
        assert torch.equal(torch.cat([t.sf[g * chunk:(g + 1) * chunk] for g in groups]).cpu(), ref["sf"])
        return ref

    xg, xrows = sample(m)
    for k, n in [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072)]:
        g = torch.Generator(device=cuda).manual_seed(k + n)
        x = torch.randn(m, k, generator=g, device=cuda)
        x = torch.where(torch.rand(m, k, generator=g, device=cuda) < 0.001, 20 * x, x)
        x[0, 5] = 1000.0
        x = x.to(torch.bfloat16)
        w = torch.randn(n, k, generator=g, device=cuda) * 0.02
        w[0, 7] = 1.0
        w = w.to(torch.bfloat16)
        bias = (torch.randn(n, generator=g, device=cuda) * 0.1).to(torch.bfloat16)
        a = ops.quant_nvfp4(x, hi_first=False)
        wq = ops.quant_nvfp4(w, hi_first=False)
        y = ops.gemm_nvfp4(a, wq, bias)

        wg, wrows = sample(n)
        a_ref = check_rows(a, x, xg, xrows, k)
        w_ref = check_rows(wq, w, wg, wrows, k)
        exact = O.nvfp4_linear_w4a4(a_ref, w_ref, k, bias[wrows.to(cuda)].cpu(), a_hi_first=False,
                                    w_hi_first=False)
        assert_close_bf16(y[xrows.to(cuda)][:, wrows.to(cuda)], exact)


def _bf16_ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()


@pytest.mark.parametrize("fmt", ["int8", "nvfp4"])
@pytest.mark.parametrize("m,ffn,k", [(200, 224, 512), (130, 1536, 3072)])
def test_swiglu_epilogue(cuda, fmt, m, ffn, k):
    """fc1 with the fused SwiGLU epilogue vs the reference's unfused chain on
    the same accumulators: STORE the [m, 2*ffn] bf16 output, then
    F.silu(gate) * up in bf16 (model/dit.py:120-129).  The two silu
    evaluations may differ in the last fp32 bit; allow 1 bf16 ulp in <0.1%."""
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.modules import QuantLinear

    g = torch.Generator().manual_seed(m + ffn)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(cuda)
    w = torch.randn(2 * ffn, k, generator=g) * 0.05
    if fmt == "int8":
        wq, ws = O.quantize_weight_int8(w)
        ql = QuantLinear.from_quant_tensors(wq, meta={"format": "int8_tensorwise"}, weight_scale=ws, device=cuda)
    else:
        qz = O.nvfp4_quantize(w.to(torch.bfloat16), hi_first=True)
        ql = QuantLinear.from_quant_tensors(qz["codes"], meta={"format": "nvfp4"}, weight_scale=qz["sf"],
                                            weight_scale_2=qz["gs"], device=cuda)
    full = ql.forward_fused(x)                       # [m, 2*ffn], reference column order
    gate, up = full.chunk(2, dim=-1)
    want = (F.silu(gate) * up)
    ql.interleave_swiglu()
    amax = torch.zeros(1, dtype=torch.float32, device=cuda)
    got = ql.forward_fused(x, epilogue=ops.EPI_SWIGLU, amax_out=amax)
    assert got.shape == (m, ffn)
    ulp = _bf16_ulps(got, want)
    assert int(ulp.max()) <= 1 and (ulp > 0).float().mean().item() < 1e-3
    assert amax.item() == got.float().abs().max().item()
    # the plain forward still returns the reference's [gate | up] column order
    assert torch.equal(ql(x), full)


@pytest.mark.parametrize("fmt", ["int8_tensorwise", "nvfp4"])
def test_quant_linear_empty_batch(cuda, fmt):
    """An empty batch gives an empty result, as F.linear does in the
    reference's fallback (int8_convrot.py:199-209): no kernel fails on zero
    rows."""
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.block import load_quant_linear
    from minixmax_h3_b200.modules import QuantLinear

    ql = QuantLinear(512, 384, bias=False, device=cuda)
    load_quant_linear(ql, torch.randn(384, 512, device=cuda) * 0.02, fmt)
    x = torch.empty(0, 512, dtype=torch.bfloat16, device=cuda)
    assert ql(x).shape == (0, 384)
    assert ql.forward_fused(x).shape == (0, 384)
    q = torch.randn(0, 2, 128, device=cuda).to(torch.bfloat16)
    kv = torch.randn(64, 2, 128, device=cuda).to(torch.bfloat16)
    assert ops.attention(q, kv, kv).shape == (0, 2, 128)
    torch.cuda.synchronize()


@pytest.mark.parametrize("fmt", ["int8_tensorwise", "nvfp4"])
def test_pre_quant_scale_on_the_fused_entry(cuda, fmt):
    """A layer with a checkpoint pre_quant_scale (modules/linear.py:184-185)
    gives, through forward_fused (the entry the block uses) and given the
    unscaled input's amax, the same bits as a layer without the scale fed
    x * pre_quant_scale; forward() agrees."""
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.block import load_quant_linear
    from minixmax_h3_b200.modules import QuantLinear

    g = torch.Generator(device=cuda).manual_seed(4)
    w = torch.randn(384, 512, generator=g, device=cuda) * 0.02
    plain = QuantLinear(512, 384, bias=False, device=cuda)
    load_quant_linear(plain, w, fmt)
    scaled = QuantLinear(512, 384, bias=False, device=cuda)
    load_quant_linear(scaled, w, fmt)
    scaled.pre_quant_scale = torch.linspace(0.25, 4.0, 512, device=cuda)
    x = torch.randn(200, 512, generator=g, device=cuda).to(torch.bfloat16)
    xs = x * scaled.pre_quant_scale.to(torch.bfloat16)
    stale_amax = ops.amax(x)
    assert torch.equal(scaled.forward_fused(x, amax=stale_amax), plain.forward_fused(xs))
    assert torch.equal(scaled(x), plain(xs))
