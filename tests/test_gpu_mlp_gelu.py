"""GPU: the GELU MLP's activation fused with fc2's NVFP4 input quantisation.

fc1 stores its bf16 output y with max(0, max y) (EPI_STORE_POSMAX); fc2's
quantiser computes u = bf16(gelu(y)) on the fly (h3b_quant_nvfp4_gelu) —
the reference's F.gelu of the bf16 linear output (model/dit.py:298-301,
ops/fused_block.py:61-63) — and takes max |u| from max y, or from
h3b_gelu_amax_scan when that bound does not settle it.  Checked bit for bit
against the two-pass path (torch's GELU on the GPU, then the plain quantiser)
and against the oracle's quantiser."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import oracle.h3_oracle as O

pytestmark = pytest.mark.gpu

NEG_BOUND = 0.169921875  # max |bf16(gelu(y))| over y < 0


def _two_pass(y):
    from minixmax_h3_b200 import ops
    u = F.gelu(y)  # bf16 in, fp32 math, bf16 out
    amax = u.abs().max().float().reshape(1)
    return u, amax, ops.quant_nvfp4(u, amax_t=amax)


def _fused(y):
    from minixmax_h3_b200 import ops
    ymax2 = torch.zeros(2, dtype=torch.float32, device=y.device)
    ymax2[0] = y.float().max().clamp(min=0.0)
    ops.gelu_amax_scan(y, ymax2)
    return ymax2, ops.quant_nvfp4_gelu(y, ymax2)


@pytest.mark.parametrize("m,k,scale", [(300, 512, 1.0), (128, 3072, 2.0), (77, 256, 0.5)])
def test_quant_nvfp4_gelu_matches_two_pass(cuda, m, k, scale):
    g = torch.Generator(device=cuda).manual_seed(m + k)
    y = (scale * torch.randn(m, k, generator=g, device=cuda)).to(torch.bfloat16)
    u, amax, ref = _two_pass(y)
    ymax2, got = _fused(y)
    assert ymax2[1].item() == 0.0  # the bound settled max |u|: no scan
    assert torch.equal(got.gs, ref.gs), (got.gs.item(), ref.gs.item())
    assert torch.equal(got.sf, ref.sf)
    assert torch.equal(got.codes, ref.codes)
    # and the quantiser itself against the oracle on the same u
    want = O.nvfp4_quantize(u.cpu(), hi_first=False, amax=amax.item())
    assert torch.equal(got.codes.cpu(), want["codes"])
    assert torch.equal(got.gs.cpu(), want["gs"])


def test_gelu_amax_scan_covers_small_outputs(cuda):
    """max y = 0.25 gives gelu = 0.148 < 0.1699: max |u| comes from the
    negative inputs (down to gelu(-0.75) = -0.17), found by the scan."""
    g = torch.Generator(device=cuda).manual_seed(5)
    y = (torch.rand(256, 512, generator=g, device=cuda) * 1.25 - 1.0).to(torch.bfloat16)  # [-1, 0.25)
    u, amax, ref = _two_pass(y)
    assert amax.item() > F.gelu(y.float().max()).item()  # the negative side sets max |u|
    ymax2, got = _fused(y)
    assert ymax2[1].item() == amax.item()
    assert torch.equal(got.gs, ref.gs)
    assert torch.equal(got.sf, ref.sf)
    assert torch.equal(got.codes, ref.codes)


def test_gelu_amax_scan_skips_when_bound_settles(cuda):
    from minixmax_h3_b200 import ops
    y = torch.full((64, 64), -0.75, dtype=torch.bfloat16, device=cuda)
    ymax2 = torch.tensor([1.0, 0.0], dtype=torch.float32, device=cuda)  # gelu(1) = 0.84 >= bound
    ops.gelu_amax_scan(y, ymax2)
    assert ymax2[1].item() == 0.0
    assert abs(F.gelu(y.float()).abs().max().item() - 0.16997) < 1e-4  # what the bound covers
    assert F.gelu(y).abs().max().item() <= NEG_BOUND


def test_store_posmax_epilogue(cuda):
    from minixmax_h3_b200 import ops
    g = torch.Generator(device=cuda).manual_seed(9)
    for m in (128, 700):  # single-CTA and CTA-pair kernels
        a = ops.quant_nvfp4(torch.randn(m, 512, generator=g, device=cuda).to(torch.bfloat16))
        w = ops.quant_nvfp4((0.05 * torch.randn(320, 512, generator=g, device=cuda)).to(torch.bfloat16))
        plain = ops.gemm_nvfp4(a, w)
        amax_pos = torch.zeros(1, dtype=torch.float32, device=cuda)
        y = ops.gemm_nvfp4(a, w, epilogue=ops.EPI_STORE_POSMAX, amax_out=amax_pos)
        assert torch.equal(y, plain)
        assert amax_pos.item() == max(0.0, plain.float().max().item())


def test_mlp_gelu_path_matches_epilogue_gelu_chain(cuda):
    """The block's GELU MLP through the fused quantiser equals fc1 with the
    GELU epilogue (same bf16(gelu(bf16 y)) chain) followed by the plain
    quantiser and fc2, bit for bit."""
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200.block import MLP, load_quant_linear

    hidden, ffn, m = 256, 1024, 300
    gen = torch.Generator().manual_seed(3)
    mlp = MLP(hidden, ffn, act="gelu", device=cuda)
    for ql, (n, k) in ((mlp.fc1, (ffn, hidden)), (mlp.fc2, (hidden, ffn))):
        load_quant_linear(ql, (torch.randn(n, k, generator=gen) * 0.05).to(cuda), "nvfp4")
    h = torch.randn(m, hidden, generator=gen).to(torch.bfloat16).to(cuda)
    out = mlp(h)
    # the same layers with fc1's GELU epilogue and the plain quantiser
    amax_u = torch.zeros(1, dtype=torch.float32, device=cuda)
    u = mlp.fc1.forward_fused(h, epilogue=ops.EPI_GELU, amax_out=amax_u)
    ref = mlp.fc2.forward_fused(u, amax=amax_u)
    assert torch.equal(out, ref)
