"""GPU: the ``torch.ops.h3b.*`` operators and the reference-named entries
(ops.int8_convrot_linear / rotate_activation, attention.gather_fa_bnsd /
sp_gather_fa / ring_attention_bnsd) give the same
bits as the ``ops`` calls and entries they wrap: the same kernels on the same
inputs, so the comparison is exact."""
from __future__ import annotations

import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(cuda, m=300, k=512, n=384, seed=0):
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    return g, x, w


def test_int8_operators(cuda):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200 import torch_ops  # noqa: F401 - registers torch.ops.h3b

    g, x, _ = _inputs(cuda)
    for group in (0, 256):
        q, s = torch.ops.h3b.quant_i8_rows(x, group)
        q_ref, s_ref = ops.quant_i8_rows(x, convrot_group=group)
        assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
    w = torch.randint(-128, 128, (384, 512), dtype=torch.int8, device=cuda, generator=g)
    ws = torch.rand(384, device=cuda, generator=g) * 1e-3
    bias = torch.randn(384, device=cuda, generator=g).to(torch.bfloat16)
    for epi in (ops.EPI_STORE, ops.EPI_GELU):
        y = torch.ops.h3b.gemm_i8(q, s, w, ws, bias, epi)
        assert torch.equal(y, ops.gemm_i8(q, s, w, ws, bias, epilogue=epi))


def test_nvfp4_operators(cuda):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200 import torch_ops  # noqa: F401

    _, x, w = _inputs(cuda, seed=1)
    c, sf, gs = torch.ops.h3b.quant_nvfp4(x, False)
    a = ops.quant_nvfp4(x, hi_first=False)
    assert torch.equal(c, a.codes) and torch.equal(sf, a.sf) and torch.equal(gs, a.gs)
    wq = ops.quant_nvfp4(w, hi_first=False)
    y = torch.ops.h3b.gemm_nvfp4(c, sf, gs, wq.codes, wq.sf, wq.gs, None, ops.EPI_STORE)
    assert torch.equal(y, ops.gemm_nvfp4(a, wq))
    # the GELU MLP's fused activation + quantisation, against the ops calls
    ymax2 = torch.zeros(2, dtype=torch.float32, device=cuda)
    ymax2[0] = y.float().max().clamp(min=0.0)
    torch.ops.h3b.gelu_amax_scan(y, ymax2)
    cg, sfg, gsg = torch.ops.h3b.quant_nvfp4_gelu(y, ymax2, False)
    ref2 = torch.zeros_like(ymax2)
    ref2[0] = ymax2[0]
    ops.gelu_amax_scan(y, ref2)
    assert torch.equal(ymax2, ref2)
    u = ops.quant_nvfp4_gelu(y, ref2)
    assert torch.equal(cg, u.codes) and torch.equal(sfg, u.sf) and torch.equal(gsg, u.gs)


def test_attention_and_norm_operators(cuda):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200 import torch_ops  # noqa: F401
    from minixmax_h3_b200.attention import h3_attention_bnsd

    g = torch.Generator(device=cuda).manual_seed(2)
    q, k, v = (torch.randn(256, 2, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(3))
    assert torch.equal(torch.ops.h3b.attention(q, k, v, None), ops.attention(q, k, v))
    qb, kb, vb = (t.permute(1, 0, 2).unsqueeze(0).contiguous() for t in (q, k, v))
    assert torch.equal(torch.ops.h3b.attention_bnsd(qb, kb, vb, 0.1), h3_attention_bnsd(qb, kb, vb, scale=0.1))

    x = torch.randn(300, 512, generator=g, device=cuda).to(torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(512, generator=g, device=cuda)).to(torch.bfloat16)
    shift = (0.1 * torch.randn(3, 512, generator=g, device=cuda)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(3, 512, generator=g, device=cuda)).to(torch.bfloat16)
    sel = torch.randint(-1, 3, (300,), dtype=torch.int32, device=cuda, generator=g)
    h = torch.ops.h3b.rmsnorm_modulate(x, wn, shift, scale, 1e-6, sel)
    assert torch.equal(h, ops.rmsnorm_modulate(x, wn, shift, scale, 1e-6, row_sel=sel))
    q8, s8 = torch.ops.h3b.rmsnorm_modulate_quant_i8(x, wn, shift, scale, 1e-6, sel, 256)
    q_ref, s_ref = ops.rmsnorm_modulate_quant_i8(x, wn, shift, scale, 1e-6, row_sel=sel, convrot_group=256)
    assert torch.equal(q8, q_ref) and torch.equal(s8, s_ref)


def test_reference_named_entries(cuda):
    from minixmax_h3_b200 import attention as A
    from minixmax_h3_b200 import ops

    g, x, _ = _inputs(cuda, seed=3)
    w = torch.randint(-128, 128, (384, 512), dtype=torch.int8, device=cuda, generator=g)
    ws = torch.rand(384, device=cuda, generator=g) * 1e-3
    x3 = x.view(3, 100, 512)
    y = ops.int8_convrot_linear(x3, w, ws)
    q, s = ops.quant_i8_rows(x, convrot_group=256)
    assert torch.equal(y, ops.gemm_i8(q, s, w, ws).view(3, 100, 384))
    rot = ops.rotate_activation(x3, 256)
    assert torch.equal(rot.view(300, 512).cpu(), O.rotate_activation_exact(x.cpu(), 256))

    q, k, v = (torch.randn(1, 2, 256, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(3))
    want = A.fusion_attention_bnsd(q, k, v)
    assert torch.equal(A.gather_fa_bnsd(q, k, v), want)
    assert torch.equal(A.sp_gather_fa(q[0], k[0], v[0]), want[0])
    assert torch.equal(A.ring_attention_bnsd(q, k, v), want)
