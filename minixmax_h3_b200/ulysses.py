"""Ulysses sequence parallelism: sequence <-> head all-to-alls.

Same contract as the reference's ops/ulysses.py:14-61: every rank holds
S/ws tokens with all heads for the projections, and all S tokens with H/ws
heads (rank r owns heads [r*H/ws, (r+1)*H/ws)) for attention; the sequence
order after the exchange is the rank order.  The transport is NCCL
``all_to_all_single`` over NVLink.  ``all_to_all_qkv`` moves the packed
[S_local, 3, H, D] projection output in ONE exchange and returns q/k/v as
strided views that the attention kernel reads in place.
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as tdist

from .dist import is_distributed, state


def all_to_all_heads(x: torch.Tensor, *, gather_seq: bool) -> torch.Tensor:
    """gather_seq=True: [S_local, H, D] -> [S, H/ws, D];
    gather_seq=False: [S, H/ws, D] -> [S_local, H, D]  (ops/ulysses.py:14-41)."""
    if not is_distributed():
        return x
    ws = state().world_size
    group = state().group
    if gather_seq:
        s_local, heads, dim = x.shape
        if heads % ws != 0:
            raise RuntimeError(f"heads={heads} not divisible by world_size={ws}")
        h_local = heads // ws
        send = x.view(s_local, ws, h_local, dim).permute(1, 0, 2, 3).contiguous()
        recv = torch.empty_like(send)
        tdist.all_to_all_single(recv, send, group=group)
        return recv.reshape(ws * s_local, h_local, dim)
    seq, h_local, dim = x.shape
    if seq % ws != 0:
        raise RuntimeError(f"seq={seq} not divisible by world_size={ws}")
    s_local = seq // ws
    send = x.contiguous().view(ws, s_local, h_local, dim)
    recv = torch.empty_like(send)
    tdist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 0, 2, 3).reshape(s_local, ws * h_local, dim)


def all_to_all_qkv(qkv: torch.Tensor, heads: int, head_dim: int
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Packed seq->head exchange of a [S_local, 3*H*D] projection output.

    Returns q, k, v as [S, H/ws, D] views of one receive buffer laid out
    [S, 3, H/ws, D] (no per-tensor copies).
    """
    s_local = qkv.shape[0]
    if not is_distributed():
        v = qkv.view(s_local, 3, heads, head_dim)
        return v[:, 0], v[:, 1], v[:, 2]
    ws = state().world_size
    if heads % ws != 0:
        raise RuntimeError(f"heads={heads} not divisible by world_size={ws}")
    hl = heads // ws
    send = qkv.view(s_local, 3, ws, hl, head_dim).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    tdist.all_to_all_single(recv, send, group=state().group)
    r = recv.view(ws * s_local, 3, hl, head_dim)
    return r[:, 0], r[:, 1], r[:, 2]


def split_range(seq_len: int) -> tuple[int, int]:
    """This rank's token range (ops/ulysses.py:44-50)."""
    ws = state().world_size
    rank = state().rank
    if seq_len % ws != 0:
        raise RuntimeError(f"seq_len={seq_len} not divisible by world_size={ws} (pad tokens)")
    chunk = seq_len // ws
    return rank * chunk, (rank + 1) * chunk


def clip_mod_segments(segments: Sequence[tuple[int, int, int]], s0: int, s1: int) -> list[tuple[int, int, int]]:
    """Restricts (a, b, row) modulation segments to [s0, s1), re-based at s0
    (ops/ulysses.py:53-61)."""
    out: list[tuple[int, int, int]] = []
    for a, b, row in segments:
        aa, bb = max(a, s0), min(b, s1)
        if aa < bb:
            out.append((aa - s0, bb - s0, row))
    return out
