"""Ulysses sequence parallelism: sequence <-> head all-to-alls.

Same contract as the reference's ops/ulysses.py:14-61: every rank holds
S/ws tokens with all heads for the projections, and all S tokens with H/ws
heads (rank r owns heads [r*H/ws, (r+1)*H/ws)) for attention; the sequence
order after the exchange is the rank order.  The sequence-parallel scheme is
an explicit argument (``SCHEMES``; ``block.Attention(seq_parallel=...)``):

* ``p2p`` (default): no separate exchange.  The QKV GEMM epilogue stores
  each output block straight into the head owner's receive buffer, and the
  attention epilogue stores each output row into the token owner's
  out-projection input, through buffers mapped by CUDA IPC
  (``PeerBuffer``).  A collective on the compute stream orders each phase.
* ``nccl``: NCCL ``all_to_all_single`` over NVLink.  ``all_to_all_qkv``
  moves the packed [S_local, 3, H, D] projection output in ONE exchange and
  returns q/k/v as strided views that the attention kernel reads in place.
* ``allgather``: the reference's production scheme (model/dit.py:200-248):
  no head exchange; K and V of all tokens are gathered once
  (``all_gather_kv``, runtime/dist.py:291-312) and every rank attends its
  own queries over all keys, all heads.
* ``ring``: K/V chunks travel around the ring and the chunk results merge
  through their log-sum-exps (``ring_attention``, ops/fa_h3.py:159-218).

``check_shapes=True`` on an exchange makes it first confirm that all ranks
send messages of one shape (``_shapes_agree``).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch
import torch.distributed as tdist

from . import ops
from ._lib import call
from .dist import is_distributed, state


SCHEMES = ("p2p", "nccl", "allgather", "ring")


def check_scheme(scheme: str) -> str:
    """Validates a sequence-parallel scheme name (one of ``SCHEMES``)."""
    if scheme not in SCHEMES:
        raise ValueError(f"seq_parallel={scheme!r}: expected one of {', '.join(SCHEMES)}")
    return scheme


class PeerBuffer:
    """A device buffer allocated on every rank of the group, with every
    peer's copy mapped into this process by CUDA IPC (ptrs[r] = rank r's
    buffer, rank order).  Creation is collective (an all-gather of the IPC
    handles), so every rank must create the same buffers in the same order."""

    def __init__(self, shape: Sequence[int], dtype: torch.dtype, device: torch.device):
        st = state()
        self.local = torch.empty(tuple(shape), dtype=dtype, device=device)
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_int64()
        call("h3b_ipc_export", self.local.data_ptr(), ctypes.cast(handle, ctypes.c_void_p), ctypes.byref(off))
        rec = torch.tensor(list(bytes(handle)) + list(int(off.value).to_bytes(8, "little")), dtype=torch.uint8,
                           device=device)
        everyone = torch.empty(st.world_size * 72, dtype=torch.uint8, device=device)
        tdist.all_gather_into_tensor(everyone, rec, group=st.group)
        raw = bytes(everyone.cpu().tolist())
        self.ptrs: list[int] = []
        self._imported: list[tuple[int, int]] = []
        for r in range(st.world_size):
            if r == st.rank:
                self.ptrs.append(self.local.data_ptr())
                continue
            h = (ctypes.c_uint8 * 64).from_buffer_copy(raw[72 * r:72 * r + 64])
            o = int.from_bytes(raw[72 * r + 64:72 * r + 72], "little")
            p = ctypes.c_void_p()
            call("h3b_ipc_import", ctypes.cast(h, ctypes.c_void_p), o, ctypes.byref(p))
            self.ptrs.append(int(p.value))
            self._imported.append((int(p.value), o))

    def close(self) -> None:
        for p, o in self._imported:
            call("h3b_ipc_close", p, o)
        self._imported.clear()


_PEER_BUFS: dict[tuple, PeerBuffer] = {}


def peer_buffer(name: str, shape: Sequence[int], dtype: torch.dtype, device: torch.device) -> PeerBuffer:
    """Cached PeerBuffer per (name, shape, dtype, device), reused across
    blocks and steps like the reference's SP buffers (runtime/dist.py:172-203)."""
    key = (name, tuple(shape), dtype, str(device))
    buf = _PEER_BUFS.get(key)
    if buf is None:
        buf = _PEER_BUFS[key] = PeerBuffer(shape, dtype, device)
    return buf


def release_peer_buffers() -> None:
    """Unmaps every peer buffer (call before destroying the process group)."""
    for buf in _PEER_BUFS.values():
        buf.close()
    _PEER_BUFS.clear()


def phase_barrier(device: torch.device, flag: Optional[torch.Tensor] = None) -> None:
    """Orders a P2P exchange: a collective on the compute stream completes on
    a rank only after every rank's preceding launches (the P2P stores into
    this rank's buffers) have completed.  `flag` (fp32 [1]) is max-reduced
    and can carry a value the step needs anyway (an amax)."""
    if flag is None:
        flag = torch.zeros(1, dtype=torch.float32, device=device)
    tdist.all_reduce(flag, op=tdist.ReduceOp.MAX, group=state().group)


def _shapes_agree(t: torch.Tensor, check: bool) -> None:
    """With ``check``: before an exchange, every rank's message (shape and
    element size) must match, else every rank raises the same RuntimeError.
    Without the check a mismatch is not a clean error: gloo aborts the
    receiving process (its pair size check ends in std::terminate) and NCCL
    moves the wrong bytes.  Costs one small all_gather per exchange, so the
    exchanges default to check=False."""
    if not check:
        return
    st = state()
    dims = list(t.shape)
    if len(dims) > 6:
        raise RuntimeError(f"_shapes_agree: {len(dims)}-d message, at most 6 dims are described")
    mine = torch.tensor([t.dim(), t.element_size()] + dims + [-1] * (6 - len(dims)), dtype=torch.int64,
                        device=t.device)
    everyone = torch.empty(st.world_size * 8, dtype=torch.int64, device=t.device)
    tdist.all_gather_into_tensor(everyone, mine, group=st.group)
    rows = everyone.view(st.world_size, 8).cpu().tolist()
    for r, row in enumerate(rows):
        if row != rows[0]:
            def desc(v):
                return f"shape {tuple(v[2:2 + v[0]])} of {v[1]}-byte elements"
            raise RuntimeError(f"exchange mismatch: rank 0 sends {desc(rows[0])}, rank {r} sends {desc(row)}")


def all_to_all_heads(x: torch.Tensor, *, gather_seq: bool, check_shapes: bool = False) -> torch.Tensor:
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
        _shapes_agree(send, check_shapes)
        recv = torch.empty_like(send)
        tdist.all_to_all_single(recv, send, group=group)
        return recv.reshape(ws * s_local, h_local, dim)
    seq, h_local, dim = x.shape
    if seq % ws != 0:
        raise RuntimeError(f"seq={seq} not divisible by world_size={ws}")
    s_local = seq // ws
    send = x.contiguous().view(ws, s_local, h_local, dim)
    _shapes_agree(send, check_shapes)
    recv = torch.empty_like(send)
    tdist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 0, 2, 3).reshape(s_local, ws * h_local, dim)


def all_to_all_qkv(qkv: torch.Tensor, heads: int, head_dim: int, *, check_shapes: bool = False
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
    _shapes_agree(send, check_shapes)
    recv = torch.empty_like(send)
    tdist.all_to_all_single(recv, send, group=state().group)
    r = recv.view(ws * s_local, 3, hl, head_dim)
    return r[:, 0], r[:, 1], r[:, 2]


def all_gather_kv(k: torch.Tensor, v: torch.Tensor, *, check_shapes: bool = False
                  ) -> tuple[torch.Tensor, torch.Tensor]:
    """[S_local, H, D] k and v of every rank -> [S, H, D] views of one gathered
    buffer, rank order = sequence order (runtime/dist.py:291-312 with
    seq_dim=0: one collective for K and V together)."""
    if not is_distributed():
        return k, v
    st = state()
    kv = torch.stack((k, v), dim=1).contiguous()  # [S_local, 2, H, D]
    _shapes_agree(kv, check_shapes)
    out = torch.empty((st.world_size * kv.shape[0],) + tuple(kv.shape[1:]), dtype=kv.dtype, device=kv.device)
    tdist.all_gather_into_tensor(out, kv, group=st.group)
    return out[:, 0], out[:, 1]


def _global_rank(group, r: int) -> int:
    return r if group is None or group is tdist.group.WORLD else tdist.get_global_rank(group, r)


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
                   out: Optional[torch.Tensor] = None, amax_out: Optional[torch.Tensor] = None,
                   attention_fn=None, merge_fn=None, check_shapes: bool = False) -> torch.Tensor:
    """Ring sequence parallelism (ops/fa_h3.py:159-218, ring_attention_lse_bnsd):
    this rank's queries q [S_local, H, D] attend to every rank's keys/values,
    which travel around the ring (rank r sends to r+1 and receives from r-1)
    one chunk per step while the chunk in hand is processed; the chunk results
    are merged through their log-sum-exps in fp32 (ops.attention_merge_lse)
    and the last merge writes out [S_local, H, D] bf16 (max |out| into
    amax_out).  K and V travel as one [S_local, 2, H, D] buffer.

    attention_fn(q, k, v, scale, out, lse) and merge_fn(acc, acc_lse, blk,
    blk_lse, first=, out=, amax_out=) default to this package's kernels; they
    are parameters so the ring logic can be exercised on CPU."""
    s_l, heads, d = q.shape
    scale = d ** -0.5 if scale is None else float(scale)
    if out is None:
        out = torch.empty(s_l, heads, d, dtype=torch.bfloat16, device=q.device)
    if attention_fn is None:
        def attention_fn(q_, k_, v_, sc, o_, lse_):
            ops.attention(q_, k_, v_, scale=sc, out=o_, lse=lse_)
    merge_fn = merge_fn or ops.attention_merge_lse
    ws = state().world_size if is_distributed() else 1
    rank = state().rank if is_distributed() else 0
    group = state().group if is_distributed() else None
    kv = torch.stack((k, v), dim=1).contiguous()  # [S_local, 2, H, D]
    if ws > 1:
        _shapes_agree(kv, check_shapes)
    recv = torch.empty_like(kv) if ws > 1 else None
    acc = torch.empty(s_l, heads, d, dtype=torch.float32, device=q.device)
    acc_lse = torch.empty(heads, s_l, dtype=torch.float32, device=q.device)
    blk = torch.empty(s_l, heads, d, dtype=torch.bfloat16, device=q.device)
    blk_lse = torch.empty(heads, s_l, dtype=torch.float32, device=q.device)
    nxt, prv = _global_rank(group, (rank + 1) % ws), _global_rank(group, (rank + ws - 1) % ws)
    reqs: list = []
    for step in range(ws):
        if step > 0:
            for r in reqs:
                r.wait()
            kv, recv = recv, kv
        reqs = []
        if step + 1 < ws:
            reqs = tdist.batch_isend_irecv([tdist.P2POp(tdist.isend, kv, nxt, group),
                                            tdist.P2POp(tdist.irecv, recv, prv, group)])
        attention_fn(q, kv[:, 0], kv[:, 1], scale, blk, blk_lse)
        last = step == ws - 1
        merge_fn(acc, acc_lse, blk, blk_lse, first=step == 0, out=out if last else None,
                 amax_out=amax_out if last else None)
    return out


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
