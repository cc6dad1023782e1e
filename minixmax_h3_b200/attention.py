"""Attention entry points with the reference's signatures.

``h3_attention_bnsd`` (ops/fa_h3.py:224-304) and ``fusion_attention_bnsd``
(ops/attention.py:100-131) take q/k/v as [B=1, H, S, D] and return
[1, H, S_q, D]; both run the tcgen05 flash-attention kernel reading the BNSD
strides in place.  There is one backend and no SDPA fallback: unsupported
inputs raise.  The reference's sequence-parallel entries are here too:
``gather_fa_bnsd`` / ``sp_gather_fa`` (K/V all-gathered, then attention) and
``ring_attention_bnsd`` (the K/V ring with log-sum-exp merges).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops


def fusion_attention_bnsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                          scale: Optional[float] = None) -> torch.Tensor:
    if q.dim() != 4:
        raise ValueError("expected 4D qkv [B, N, S, D]")
    if q.shape[0] != 1:
        raise ValueError("batch must be 1 (the reference's DiT runs B=1, model/dit.py:765-766)")
    d = q.shape[-1]
    scale = d ** -0.5 if scale is None else scale
    qt = q[0].permute(1, 0, 2)  # [S, H, D] view of BNSD storage
    kt = k[0].permute(1, 0, 2)
    vt = v[0].permute(1, 0, 2)
    if kt.stride() != vt.stride():
        kt, vt = kt.contiguous(), vt.contiguous()
    out = torch.empty((1, q.shape[1], q.shape[2], d), dtype=torch.bfloat16, device=q.device)
    ops.attention(qt, kt, vt, scale=scale, out=out[0].permute(1, 0, 2))
    return out


def h3_attention_bnsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
                      gathered: bool = False) -> torch.Tensor:
    """Entry for the DiT: q/k/v [1, H, S, D]; ``gathered`` (KV already global)
    only matters to the reference's ring backend and is accepted for parity."""
    del gathered
    return fusion_attention_bnsd(q, k, v, scale=scale)


def _tokens(t: torch.Tensor) -> torch.Tensor:
    """[1, H, S, D] or [H, S, D] (BNSD) -> a [S, H, D] token-major view."""
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError("batch must be 1 (the reference's DiT runs B=1, model/dit.py:765-766)")
        t = t[0]
    if t.dim() != 3:
        raise ValueError("expected [1, H, S, D] or [H, S, D]")
    return t.permute(1, 0, 2)


def gather_fa_bnsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
                   gathered: bool = False) -> torch.Tensor:
    """ops/gather_fa.py:130-181: this rank's queries [1, H, Sq, D] attend over
    every rank's keys.  Unless ``gathered``, the local K/V shards ([1, H, Sk, D]
    or [H, Sk, D]) are first all-gathered along the sequence in rank order
    (ulysses.all_gather_kv).  One attention kernel serves every
    ``H3_GATHER_FA_MODE`` of the reference (its tiled and head-chunked modes
    exist to fit NPU memory).  Returns [1, H, Sq, D] bf16."""
    from .dist import is_distributed
    from .ulysses import all_gather_kv

    qt, kt, vt = _tokens(q), _tokens(k), _tokens(v)
    if not gathered and is_distributed():
        kt, vt = all_gather_kv(kt.contiguous(), vt.contiguous())
    elif kt.stride() != vt.stride():
        kt, vt = kt.contiguous(), vt.contiguous()
    s_q, heads, d = qt.shape
    out = torch.empty((1, heads, s_q, d), dtype=torch.bfloat16, device=q.device)
    ops.attention(qt, kt, vt, scale=scale, out=out[0].permute(1, 0, 2))
    return out


def sp_gather_fa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                 scale: Optional[float] = None) -> torch.Tensor:
    """ops/gather_fa.py:184-192: the DiT's gathered-attention entry on
    [H, S_local, D] q/k/v; returns [H, S_local, D]."""
    return gather_fa_bnsd(q.unsqueeze(0), k, v, scale=scale, gathered=False)[0]


def ring_attention_bnsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                        scale: Optional[float] = None) -> torch.Tensor:
    """ops/ring_attention.py:67-123: local shards [1, H, S_local, D] in, the
    same shape out.  Under a process group the K/V shards travel around the
    ring and the chunk results merge through their log-sum-exps
    (ulysses.ring_attention); on one process it is plain attention."""
    from .dist import is_distributed
    from .ulysses import ring_attention

    if not is_distributed():
        return fusion_attention_bnsd(q, k, v, scale=scale)
    o = ring_attention(_tokens(q), _tokens(k), _tokens(v), scale=scale)
    return o.permute(1, 0, 2).unsqueeze(0).contiguous()
