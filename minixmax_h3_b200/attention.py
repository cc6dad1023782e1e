"""Attention entry points with the reference's signatures.

``h3_attention_bnsd`` (ops/fa_h3.py:224-304) and ``fusion_attention_bnsd``
(ops/attention.py:100-131) take q/k/v as [B=1, H, S, D] and return
[1, H, S_q, D]; both run the tcgen05 flash-attention kernel reading the BNSD
strides in place.  There is one backend (no env-driven dispatch) and no SDPA
fallback: unsupported inputs raise.
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
        vt = vt.contiguous() if vt.is_contiguous() else vt
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
