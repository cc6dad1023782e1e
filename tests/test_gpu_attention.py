"""GPU parity: tcgen05 flash attention and the fused q/k RMSNorm + RoPE.

Bar (attention): helpers.assert_close_bf16 — scaled max-abs <= 2e-2 and
cosine >= 0.9995 against fp32 softmax attention on the CPU."""
from __future__ import annotations

import math

import pytest
import torch

from helpers import assert_close_bf16, load_golden
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu


def _ref_tokens_major(q, k, v, scale=None):
    """q/k/v [S, H, D] -> fp32 oracle output [S, H, D]."""
    return O.attention_fp32(q.permute(1, 0, 2), k.permute(1, 0, 2), v.permute(1, 0, 2), scale).permute(1, 0, 2)


def test_attention_golden_bnsd(cuda):
    from minixmax_h3_b200 import ops

    g = load_golden("attention.pt")
    q, k, v = (g[n][0].to(cuda) for n in ("q", "k", "v"))  # [H, S, D] (BNSD, B=1)
    o = torch.empty_like(q)
    ops.attention(q.permute(1, 0, 2), k.permute(1, 0, 2), v.permute(1, 0, 2), out=o.permute(1, 0, 2))
    assert_close_bf16(o, O.attention_fp32(g["q"][0], g["k"][0], g["v"][0]))
    assert_close_bf16(o, g["out"][0])  # the reference's own SDPA result


@pytest.mark.parametrize("s_q,s_kv,heads", [(128, 128, 1), (256, 1000, 3), (1000, 4096, 2), (300, 77, 2),
                                            (1, 129, 1)])
def test_attention_shapes(cuda, s_q, s_kv, heads):
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(s_q * 7 + s_kv)
    q = torch.randn(s_q, heads, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(s_kv, heads, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(s_kv, heads, 128, generator=g).to(torch.bfloat16)
    lse = torch.empty(heads, s_q, device=cuda)
    o = ops.attention(q.to(cuda), k.to(cuda), v.to(cuda), lse=lse)
    assert_close_bf16(o, _ref_tokens_major(q, k, v))
    logits = torch.einsum("shd,thd->hst", q.float(), k.float()) / math.sqrt(128)
    assert torch.allclose(lse.cpu(), torch.logsumexp(logits, dim=-1), atol=1e-3, rtol=1e-4)


def test_attention_packed_qkv_layout(cuda):
    """q/k/v read in place from a [S, 3, H, D] projection output (no copies)."""
    from minixmax_h3_b200 import ops

    s, heads = 700, 3
    qkv = torch.randn(s, 3, heads, 128, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    d = qkv.to(cuda)
    out = torch.empty(s, heads * 128, dtype=torch.bfloat16, device=cuda)
    ops.attention(d[:, 0], d[:, 1], d[:, 2], out=out.view(s, heads, 128))
    assert_close_bf16(out.view(s, heads, 128), _ref_tokens_major(qkv[:, 0], qkv[:, 1], qkv[:, 2]))


@pytest.mark.parametrize("sigma", [3.0, 6.0])
def test_attention_rescaling_stress(cuda, sigma):
    """Large, growing logits force many running-max corrections."""
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(int(sigma))
    s_q, s_kv, heads = 256, 2048, 2
    q = (torch.randn(s_q, heads, 128, generator=g) * sigma).to(torch.bfloat16)
    ramp = torch.linspace(0.2, 1.5, s_kv)[:, None, None]
    k = (torch.randn(s_kv, heads, 128, generator=g) * sigma * ramp).to(torch.bfloat16)
    v = torch.randn(s_kv, heads, 128, generator=g).to(torch.bfloat16)
    o = ops.attention(q.to(cuda), k.to(cuda), v.to(cuda))
    assert_close_bf16(o, _ref_tokens_major(q, k, v))


def test_attention_cfg4_full_size_sampled(cuda):
    """BASELINE cfg 4 single-GPU shape: S=131072, 24 heads; 128 query rows of
    two heads re-derived on the CPU against the full K/V."""
    from minixmax_h3_b200 import ops

    s, heads = 131072, 24
    gen = torch.Generator(device=cuda).manual_seed(0)
    q = torch.randn(s, heads, 128, generator=gen, device=cuda).to(torch.bfloat16)
    k = torch.randn(s, heads, 128, generator=gen, device=cuda).to(torch.bfloat16)
    v = torch.randn(s, heads, 128, generator=gen, device=cuda).to(torch.bfloat16)
    o = ops.attention(q, k, v)
    rows = torch.randperm(s, generator=torch.Generator().manual_seed(1))[:128].to(cuda)
    for h in (0, 23):
        want = O.attention_fp32(q[rows, h][None].cpu(), k[:, h][None].cpu(), v[:, h][None].cpu())[0]
        assert_close_bf16(o[rows, h], want)


def test_qk_rmsnorm_rope_golden(cuda):
    from minixmax_h3_b200 import ops

    g = load_golden("rope.pt")
    q = g["q"][0].to(cuda).clone()  # [S, H, D]
    ops.qk_rmsnorm_rope(q, None, g["weight"].to(cuda), None, g["eps"], g["pos"].to(cuda), 0,
                        g["inv_freq"].to(cuda), g["n_t"], g["n_h"])
    want = g["out"][0]
    diff = (q.cpu().float() - want.float()).abs()
    # bf16 arithmetic as in the reference; cos/sin may differ from the CPU
    # libm in the last fp32 bit, which can flip a bf16 rounding of the table
    assert (diff > 0).float().mean().item() < 2e-3
    assert_close_bf16(q, want, max_abs=1e-2)


def test_qk_rmsnorm_rope_q_and_k_with_offset(cuda):
    from minixmax_h3_b200 import ops

    grid = (4, 6, 8)
    pos = O.grid_positions(*grid)
    s_total, heads, off, s_loc = pos.shape[0], 2, 48, 96
    gen = torch.Generator().manual_seed(3)
    qkv = torch.randn(s_loc, 3, heads, 128, generator=gen).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    inv = O.rope_inv_freq()
    d = qkv.to(cuda)
    ops.qk_rmsnorm_rope(d[:, 0], d[:, 1], qw.to(cuda), kw.to(cuda), 1e-6, pos.to(cuda), off, inv.to(cuda), 22, 21)
    table = O.rope_rotation_table(O.rope_angles(pos[off:off + s_loc], inv, 22, 21), torch.bfloat16)
    want_q = O.rms_rope_apply(qkv[:, 0][None], table, qw, 1e-6, 128)[0]
    want_k = O.rms_rope_apply(qkv[:, 1][None], table, kw, 1e-6, 128)[0]
    assert_close_bf16(d[:, 0], want_q, max_abs=1e-2)
    assert_close_bf16(d[:, 1], want_k, max_abs=1e-2)
    assert torch.equal(d[:, 2].cpu(), qkv[:, 2])  # v untouched


def test_rmsnorm_modulate_and_gate(cuda):
    from minixmax_h3_b200 import ops

    gen = torch.Generator().manual_seed(4)
    m, hidden = 515, 3072
    x = torch.randn(m, hidden, generator=gen).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=gen)).to(torch.bfloat16)
    shift = (0.1 * torch.randn(hidden, generator=gen)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(hidden, generator=gen)).to(torch.bfloat16)
    amax = torch.zeros(1, device=cuda)
    h = ops.rmsnorm_modulate(x.to(cuda), w.to(cuda), shift.to(cuda), scale.to(cuda), 1e-6, amax_out=amax)
    want = O.mod_scale_shift(O.rms_norm(x, w, 1e-6), shift[None], scale[None], [(0, m, 0)])
    assert_close_bf16(h, want, max_abs=1e-2)
    assert amax.item() == h.float().abs().max().item()
    y = torch.randn(m, hidden, generator=gen).to(torch.bfloat16)
    gate = torch.randn(hidden, generator=gen).to(torch.bfloat16)
    xd = x.to(cuda)
    ops.gate_residual(xd, y.to(cuda), gate.to(cuda))
    want_x = O.mod_gate(x.clone(), gate[None], y, [(0, m, 0)])
    assert_close_bf16(xd, want_x, max_abs=1e-2)


# ---------------------------------------------------------------- LSE merge (ring SP)

def test_merge_lse_kernel_matches_reference_formula(cuda):
    """h3b_attention_merge_lse vs ops/fa_h3.py:141-156 restated in fp32."""
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(11)
    s, heads = 333, 3
    acc = torch.randn(s, heads, 128, generator=g)
    blk = torch.randn(s, heads, 128, generator=g).to(torch.bfloat16)
    acc_lse = torch.randn(heads, s, generator=g) * 4
    blk_lse = torch.randn(heads, s, generator=g) * 4
    a, al = acc.to(cuda), acc_lse.to(cuda)
    ops.attention_merge_lse(a, al, blk.to(cuda), blk_lse.to(cuda), first=False)
    want_o, want_l = O.merge_lse(acc, acc_lse, blk, blk_lse)
    assert torch.allclose(a.cpu(), want_o, atol=1e-5, rtol=1e-5)
    assert torch.allclose(al.cpu(), want_l, atol=1e-5, rtol=1e-6)
    # final merge: bf16 out and its |max|, acc untouched
    a2, al2 = acc.to(cuda), acc_lse.to(cuda)
    out = torch.empty(s, heads, 128, dtype=torch.bfloat16, device=cuda)
    amax = torch.zeros(1, device=cuda)
    ops.attention_merge_lse(a2, al2, blk.to(cuda), blk_lse.to(cuda), first=False, out=out, amax_out=amax)
    assert torch.equal(a2.cpu(), acc)
    assert torch.allclose(out.float().cpu(), want_o, atol=2e-2, rtol=1e-2)
    assert amax.item() == out.float().abs().max().item()
    # first: plain copy
    ops.attention_merge_lse(a, al, blk.to(cuda), blk_lse.to(cuda), first=True)
    assert torch.equal(a.cpu(), blk.float()) and torch.equal(al.cpu(), blk_lse)


@pytest.mark.parametrize("chunks", [2, 3])
def test_chunked_attention_with_lse_merge(cuda, chunks):
    """Attention over K/V split into chunks, merged through the LSEs (the ring
    step, here on one GPU), against attention over the whole K/V."""
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(chunks)
    s_q, s_kv, heads = 300, 384 * chunks, 2
    q = torch.randn(s_q, heads, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(s_kv, heads, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(s_kv, heads, 128, generator=g).to(torch.bfloat16).to(cuda)
    acc = torch.empty(s_q, heads, 128, device=cuda)
    acc_lse = torch.empty(heads, s_q, device=cuda)
    blk = torch.empty(s_q, heads, 128, dtype=torch.bfloat16, device=cuda)
    blk_lse = torch.empty(heads, s_q, device=cuda)
    out = torch.empty_like(blk)
    c = s_kv // chunks
    for i in range(chunks):
        ops.attention(q, k[i * c:(i + 1) * c], v[i * c:(i + 1) * c], out=blk, lse=blk_lse)
        ops.attention_merge_lse(acc, acc_lse, blk, blk_lse, first=i == 0, out=out if i == chunks - 1 else None)
    full_lse = torch.empty(heads, s_q, device=cuda)
    full = ops.attention(q, k, v, lse=full_lse)
    assert torch.allclose(acc_lse, full_lse, atol=1e-4, rtol=1e-5)
    assert_close_bf16(out, _ref_tokens_major(q.cpu(), k.cpu(), v.cpu()))
    g_, w_ = out.float().reshape(-1), full.float().reshape(-1)
    assert torch.nn.functional.cosine_similarity(g_, w_, dim=0).item() > 0.9999
