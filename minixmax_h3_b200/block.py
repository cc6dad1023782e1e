"""DiT block on the B200 kernels, with the reference's module surface.

Mirrors model/dit.py of the reference: ``Attention`` (156-289), ``MLP``
(291-301), ``AdalnProj`` (304-329), ``_mod_scale_shift``/``_mod_gate``
(332-341) and ``DiTBlock`` (400-449), same constructor arguments and
``forward(x, t_emb, mod_segments, rope_freqs)``.  The forward is one fused
pipeline per sublayer:

    rmsnorm+modulate(+|h| max) -> quantise -> QKV GEMM -> q/k RMSNorm+RoPE
    -> [Ulysses seq->head] -> flash attention(+|o| max) -> [head->seq]
    -> quantise -> out-proj GEMM with the gate*y + x residual in its epilogue
    rmsnorm+modulate(+max) -> quantise -> fc1 GEMM (+GELU, +max)
    -> quantise -> fc2 GEMM with the gate residual in its epilogue

``rope_freqs`` is a ``RopeSpec`` (grid positions + inverse frequencies); the
kernels build the reference's bf16 rotation table (ops/rope.py:7-13) on the
fly instead of reading a [1, S, 1, 64, 2, 2] table.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .dist import is_distributed, state
from .modules import Linear, Ops, QuantizedRows, QuantLinear, RMSNorm
from .ops import EPI_GATE_RES, EPI_GELU, EPI_STORE_POSMAX, EPI_SWIGLU
from .timing import TIMER
from .ulysses import (all_gather_kv, all_to_all_heads, all_to_all_qkv, check_scheme, clip_mod_segments,
                      peer_buffer, phase_barrier, ring_attention, split_range)


@dataclass
class RopeSpec:
    """3D RoPE inputs: ``pos`` [S_total, 3] fp32 (t, h, w) per token of the
    whole (unsharded) sequence, ``inv_freq`` [64] fp32 laid out t|h|w with
    n_t / n_h entries for the t / h axes (model/dit.py:746-752)."""

    pos: torch.Tensor
    inv_freq: torch.Tensor
    n_t: int
    n_h: int

    @staticmethod
    def inv_freq_for(dims: Sequence[int] = (44, 42, 42), theta: float = 10000.0) -> torch.Tensor:
        parts = [1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d)) for d in dims]
        return torch.cat(parts)

    @classmethod
    def build(cls, pos: torch.Tensor, dims: Sequence[int] = (44, 42, 42), device=None) -> "RopeSpec":
        if sum(dims) != 128:
            raise ValueError("rope axis dims must sum to the head dim (128)")
        inv = cls.inv_freq_for(dims)
        return cls(pos.to(device=device, dtype=torch.float32).contiguous(), inv.to(device), dims[0] // 2,
                   dims[1] // 2)

    @staticmethod
    def grid_positions(t: int, h: int, w: int) -> torch.Tensor:
        tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
        return torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], dim=-1).to(torch.float32)


def global_amax_(amax: Optional[torch.Tensor], ql: QuantLinear) -> Optional[torch.Tensor]:
    """Makes an NVFP4 activation's global scale independent of the GPU count:
    under sequence parallelism each rank sees only its tokens, so the |x| max
    feeding gs = amax/(6*448) is max-reduced across ranks (one float) before
    the quantiser runs.  INT8 scales are per token and need nothing."""
    if amax is not None and ql.quant_format == "nvfp4" and is_distributed():
        import torch.distributed as tdist

        with TIMER.span("amax_allreduce"):
            tdist.all_reduce(amax, op=tdist.ReduceOp.MAX, group=state().group)
    return amax


def segments_to_row_sel(segments: Sequence[tuple[int, int, int]], s_len: int, device) -> torch.Tensor:
    """Per-token adaLN row index for (a, b, row) segments; -1 = no segment
    (such tokens are normalised but neither modulated nor gated, exactly as
    the reference's per-segment in-place updates leave them)."""
    sel = torch.full((s_len,), -1, dtype=torch.int32)
    for a, b, row in segments:
        sel[a:b] = int(row)
    return sel.to(device, non_blocking=True)


class AdalnProj(nn.Module):
    """model/dit.py:304-329: linear(silu?(t_emb)) -> `expand` chunks, each a
    [rows*modalities, hidden] view (row stride expand*hidden, no copies)."""

    def __init__(self, t_dim, hidden, expand, modalities, apply_silu=True, dtype=None, device=None,
                 operations=None):
        super().__init__()
        operations = operations or Ops
        self.expand = expand
        self.modalities = modalities
        self.hidden = hidden
        self.apply_silu = apply_silu
        self.linear = operations.Linear(t_dim, expand * hidden * modalities, bias=True, dtype=dtype, device=device)

    def forward(self, t_emb):
        x = self.linear(F.silu(t_emb) if self.apply_silu else t_emb)
        x = x.to(torch.bfloat16).reshape(x.shape[0] * self.modalities, self.expand * self.hidden)
        return x.chunk(self.expand, dim=-1)


class Attention(nn.Module):
    """model/dit.py:156-289.  Under a process group (``sequence_parallel``)
    the attention runs Ulysses-sharded with the exchange scheme
    ``seq_parallel`` (one of ``ulysses.SCHEMES``: "p2p" fused P2P stores,
    "nccl" all-to-alls, "allgather" K/V gather, "ring" K/V ring)."""

    def __init__(self, hidden, heads, head_dim, eps, dtype=None, device=None, operations=None,
                 sequence_parallel=True, seq_parallel: str = "p2p"):
        super().__init__()
        operations = operations or Ops
        if head_dim != 128:
            raise ValueError("the attention kernel is specialised for head_dim 128")
        self.heads = heads
        self.head_dim = head_dim
        self.sequence_parallel = sequence_parallel
        self.seq_parallel = check_scheme(seq_parallel)
        inner = heads * head_dim
        self.qkv_proj = operations.QuantLinear(hidden, inner * 3, bias=False, dtype=dtype, device=device)
        self.q_norm = operations.RMSNorm(head_dim, eps=eps, dtype=dtype, device=device)
        self.k_norm = operations.RMSNorm(head_dim, eps=eps, dtype=dtype, device=device)
        self.out_proj = operations.QuantLinear(inner, hidden, bias=False, dtype=dtype, device=device)

    def forward(self, h: torch.Tensor, rope_freqs: Optional[RopeSpec] = None, *, amax_h=None, resid=None,
                gate=None, row_sel=None) -> torch.Tensor:
        """h [S_local, hidden] bf16.  With resid/gate given, returns resid
        updated in place by resid += gate[row_sel] * attn(h) (fused epilogue);
        otherwise returns attn(h)."""
        s_local = h.shape[0]
        sp = self.sequence_parallel and is_distributed()
        if sp and self.seq_parallel == "p2p":
            return self._forward_p2p(h, rope_freqs, amax_h=amax_h, resid=resid, gate=gate, row_sel=row_sel)
        gather_kv = sp and self.seq_parallel == "allgather"
        ring = sp and self.seq_parallel == "ring"
        qkv = self.qkv_proj.forward_fused(h, amax=global_amax_(amax_h, self.qkv_proj))  # [S_l, 3*H*D]
        q3 = qkv.view(s_local, 3, self.heads, self.head_dim)
        with TIMER.span("rope"):
            if rope_freqs is not None:
                s0 = split_range(rope_freqs.pos.shape[0])[0] if sp else 0
                ops.qk_rmsnorm_rope(q3[:, 0], q3[:, 1], self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
                                    rope_freqs.pos, s0, rope_freqs.inv_freq, rope_freqs.n_t, rope_freqs.n_h)
            else:
                # q/k RMSNorm only (RoPE-free blocks): fold into the rope kernel
                # with zero frequencies (cos 1, sin 0).
                zeros = torch.zeros(64, dtype=torch.float32, device=h.device)
                pos0 = torch.zeros(s_local, 3, dtype=torch.float32, device=h.device)
                ops.qk_rmsnorm_rope(q3[:, 0], q3[:, 1], self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
                                    pos0, 0, zeros, 64, 0)
        amax_o = torch.zeros(1, dtype=torch.float32, device=h.device)
        if ring:
            # ring SP (ops/fa_h3.py:159-218): local queries, K/V chunks passed
            # around the ring, chunk results merged through their LSEs
            flops = 4.0 * s_local * s_local * state().world_size * self.head_dim * self.heads
            with TIMER.span("attention", flops):
                o = ring_attention(q3[:, 0], q3[:, 1], q3[:, 2], scale=self.head_dim ** -0.5, amax_out=amax_o)
            o = o.view(s_local, self.heads * self.head_dim)
            global_amax_(amax_o, self.out_proj)
        elif gather_kv:
            # the reference's production SP (model/dit.py:200-248): local
            # queries over the gathered keys/values of all ranks, all heads
            with TIMER.span("exchange"):
                k, v = all_gather_kv(q3[:, 1], q3[:, 2])
            flops = 4.0 * s_local * k.shape[0] * self.head_dim * self.heads
            with TIMER.span("attention", flops):
                o = ops.attention(q3[:, 0], k, v, scale=self.head_dim ** -0.5, amax_out=amax_o)
            o = o.view(s_local, self.heads * self.head_dim)
            global_amax_(amax_o, self.out_proj)
        elif sp:
            with TIMER.span("exchange"):
                q, k, v = all_to_all_qkv(qkv, self.heads, self.head_dim)
            flops = 4.0 * q.shape[0] * k.shape[0] * self.head_dim * q.shape[1]
            with TIMER.span("attention", flops):
                o = ops.attention(q, k, v, scale=self.head_dim ** -0.5)
            with TIMER.span("exchange"):
                o = all_to_all_heads(o, gather_seq=False).reshape(s_local, self.heads * self.head_dim)
                o = o.contiguous()
            ops.amax(o, out=amax_o)
            global_amax_(amax_o, self.out_proj)
        else:
            flops = 4.0 * s_local * s_local * self.head_dim * self.heads
            with TIMER.span("attention", flops):
                o = ops.attention(q3[:, 0], q3[:, 1], q3[:, 2], scale=self.head_dim ** -0.5, amax_out=amax_o)
            o = o.view(s_local, self.heads * self.head_dim)
        if resid is not None:
            return self.out_proj.forward_fused(o, amax=amax_o, epilogue=EPI_GATE_RES, resid=resid, gate=gate,
                                               row_sel=row_sel)
        return self.out_proj.forward_fused(o, amax=amax_o)

    def _forward_p2p(self, h: torch.Tensor, rope_freqs: Optional[RopeSpec], *, amax_h=None, resid=None,
                     gate=None, row_sel=None) -> torch.Tensor:
        """Sequence-parallel attention with both Ulysses exchanges fused into
        kernels: the QKV GEMM stores into the head owners' receive buffers, the
        attention stores into the token owners' out-projection inputs.  Each
        phase ends with a collective on the compute stream (see
        ulysses.phase_barrier); RMSNorm + RoPE run after the exchange on the
        full sequence (per-token, per-head: the same values as before it)."""
        st = state()
        ws, rank = st.world_size, st.rank
        s_local = h.shape[0]
        hl = self.heads // ws
        s_full = s_local * ws
        recv = peer_buffer("ulysses_qkv", (s_full, 3, hl, self.head_dim), torch.bfloat16, h.device)
        obuf = peer_buffer("ulysses_o", (s_local, self.heads, self.head_dim), torch.bfloat16, h.device)
        self.qkv_proj.forward_seq2head(h, recv.ptrs, rank, self.heads, amax=global_amax_(amax_h, self.qkv_proj))
        with TIMER.span("phase_barrier"):
            phase_barrier(h.device)
        q, k, v = recv.local[:, 0], recv.local[:, 1], recv.local[:, 2]
        with TIMER.span("rope"):
            if rope_freqs is not None:
                ops.qk_rmsnorm_rope(q, k, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps, rope_freqs.pos,
                                    0, rope_freqs.inv_freq, rope_freqs.n_t, rope_freqs.n_h)
            else:
                zeros = torch.zeros(64, dtype=torch.float32, device=h.device)
                pos0 = torch.zeros(s_full, 3, dtype=torch.float32, device=h.device)
                ops.qk_rmsnorm_rope(q, k, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps, pos0, 0, zeros,
                                    64, 0)
        amax_o = torch.zeros(1, dtype=torch.float32, device=h.device)
        flops = 4.0 * s_full * s_full * self.head_dim * hl
        with TIMER.span("attention", flops):
            ops.attention_head2seq(q, k, v, obuf.ptrs, s_local=s_local, head0=rank * hl, total_heads=self.heads,
                                   scale=self.head_dim ** -0.5, amax_out=amax_o)
        with TIMER.span("phase_barrier"):
            phase_barrier(h.device, amax_o)  # orders the O stores; amax_o is now the global max
        o = obuf.local.view(s_local, self.heads * self.head_dim)
        if resid is not None:
            return self.out_proj.forward_fused(o, amax=amax_o, epilogue=EPI_GATE_RES, resid=resid, gate=gate,
                                               row_sel=row_sel)
        return self.out_proj.forward_fused(o, amax=amax_o)


class MLP(nn.Module):
    """fc1 -> activation -> fc2 (model/dit.py:291-301).  act="swiglu" is the
    reference MLP (fc1: hidden -> 2*ffn, silu(gate)*up, fused into fc1's
    epilogue); act="gelu" is the benchmark's 4x GELU MLP (fc1: hidden -> ffn,
    exact-erf GELU of fc1's bf16 output applied inside fc2's NVFP4 input
    quantiser; fused into fc1's epilogue when fc2 is INT8 or has a
    pre_quant_scale)."""

    def __init__(self, hidden, ffn, dtype=None, device=None, operations=None, act: str = "swiglu"):
        super().__init__()
        operations = operations or Ops
        if act not in ("swiglu", "gelu"):
            raise ValueError(act)
        self.act = act
        self.fc1 = operations.QuantLinear(hidden, ffn * 2 if act == "swiglu" else ffn, bias=False, dtype=dtype,
                                          device=device)
        self.fc2 = operations.QuantLinear(ffn, hidden, bias=False, dtype=dtype, device=device)

    def forward(self, h: torch.Tensor, *, amax_h=None, resid=None, gate=None, row_sel=None) -> torch.Tensor:
        amax_u = torch.zeros(1, dtype=torch.float32, device=h.device)
        amax_h = global_amax_(amax_h, self.fc1)
        if self.act == "gelu" and self.fc2.quant_format == "nvfp4" and self.fc2.pre_quant_scale is None:
            # fc1 stores its bf16 output y and max(0, max y); GELU runs inside
            # fc2's NVFP4 input quantiser, u = bf16(gelu(y)) as the reference's
            # F.gelu of the bf16 linear output.  max |u| follows from max y
            # (a scan covers the case the bound does not settle).
            ymax2 = torch.zeros(2, dtype=torch.float32, device=h.device)
            y = self.fc1.forward_fused(h, amax=amax_h, epilogue=EPI_STORE_POSMAX, amax_out=ymax2[:1])
            with TIMER.span("quant"):
                ops.gelu_amax_scan(y, ymax2)
            global_amax_(ymax2, self.fc2)
            if resid is not None:
                return self.fc2.forward_gelu_input(y, ymax2, epilogue=EPI_GATE_RES, resid=resid, gate=gate,
                                                   row_sel=row_sel)
            return self.fc2.forward_gelu_input(y, ymax2)
        if self.act == "gelu":
            u = self.fc1.forward_fused(h, amax=amax_h, epilogue=EPI_GELU, amax_out=amax_u)
        else:
            # silu(gate) * up fused into the fc1 epilogue over the interleaved weight
            self.fc1.interleave_swiglu()
            u = self.fc1.forward_fused(h, amax=amax_h, epilogue=EPI_SWIGLU, amax_out=amax_u)
        global_amax_(amax_u, self.fc2)
        if resid is not None:
            return self.fc2.forward_fused(u, amax=amax_u, epilogue=EPI_GATE_RES, resid=resid, gate=gate,
                                          row_sel=row_sel)
        return self.fc2.forward_fused(u, amax=amax_u)


class DiTBlock(nn.Module):
    """model/dit.py:400-449 on the fused kernels."""

    def __init__(self, hidden, heads, head_dim, ffn, t_dim, eps, qk_eps, apply_silu=True, adaln_dtype=None,
                 dtype=None, device=None, operations=None, mlp_act: str = "swiglu", seq_parallel: str = "p2p"):
        super().__init__()
        operations = operations or Ops
        self.hidden = hidden
        self.norm1 = operations.RMSNorm(hidden, eps=eps, dtype=dtype, device=device)
        self.norm2 = operations.RMSNorm(hidden, eps=eps, dtype=dtype, device=device)
        self.attn = Attention(hidden, heads, head_dim, qk_eps, dtype=dtype, device=device, operations=operations,
                              seq_parallel=seq_parallel)
        self.mlp = MLP(hidden, ffn, dtype=dtype, device=device, operations=operations, act=mlp_act)
        self.adaln_proj = AdalnProj(t_dim, hidden, 6, 3, apply_silu=apply_silu,
                                    dtype=adaln_dtype if adaln_dtype is not None else dtype, device=device,
                                    operations=operations)
        self._sel_cache: dict = {}

    def _row_sel(self, segments, s_len, device) -> torch.Tensor:
        key = (tuple(tuple(int(v) for v in seg) for seg in segments), s_len, str(device))
        sel = self._sel_cache.get(key)
        if sel is None:
            sel = segments_to_row_sel(segments, s_len, device)
            self._sel_cache = {key: sel}
        return sel

    def forward(self, x, t_emb, mod_segments, rope_freqs: Optional[RopeSpec] = None):
        """x [S_local, hidden] bf16, updated in place and returned (as the
        reference's in-place _mod_gate does).  Under Ulysses, mod_segments are
        already clipped to this rank (ops/ulysses.py:53-61)."""
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise TypeError("DiTBlock expects a CUDA bf16 [S, hidden] input")
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(t_emb)
        sel = self._row_sel(mod_segments, x.shape[0], x.device)
        amax = torch.zeros(2, dtype=torch.float32, device=x.device)
        h = None
        for i, (norm, shift, scale, gate, sub, ql) in enumerate((
                (self.norm1, shift_msa, scale_msa, gate_msa, self.attn, self.attn.qkv_proj),
                (self.norm2, shift_mlp, scale_mlp, gate_mlp, self.mlp, self.mlp.fc1))):
            if ql.quant_format == "int8_tensorwise" and ql.pre_quant_scale is None:
                # norm + modulate + (ConvRot) + row quantisation in one kernel
                # (a pre_quant_scale applies between the two: the layer does it)
                group = ql.group_size if ql.convrot else 0
                with TIMER.span("norm"):
                    q, xs = ops.rmsnorm_modulate_quant_i8(
                        x, norm.weight, shift, scale, norm.eps, row_sel=sel, convrot_group=group,
                        q_out=h.q if isinstance(h, QuantizedRows) else None,
                        scale_out=h.scale if isinstance(h, QuantizedRows) else None)
                h = QuantizedRows(q, xs, group)
            else:
                with TIMER.span("norm"):
                    h = ops.rmsnorm_modulate(x, norm.weight, shift, scale, norm.eps, row_sel=sel,
                                             amax_out=amax[i:i + 1], out=h if isinstance(h, torch.Tensor) else None)
            if i == 0:
                sub(h, rope_freqs, amax_h=amax[0:1], resid=x, gate=gate, row_sel=sel)
            else:
                sub(h, amax_h=amax[1:2], resid=x, gate=gate, row_sel=sel)
        return x


# ----------------------------------------------------------------------------- weights / harness


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    """[cos(t*f), sin(t*f)], f_i = max_period^(-i/(dim/2)): the benchmark's
    256-d sinusoidal timestep embedding."""
    half = dim // 2
    f = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    a = t.float()[:, None] * f[None]
    return torch.cat([torch.cos(a), torch.sin(a)], dim=-1)


def curve_t_embedding(adaln_t_table: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    """The timestep embedding of the production checkpoints (model/dit.py:
    870-874): each t in [0, 1] (clamped) lands at position t * (grid - 1) of
    the learned [grid, t_dim] ``adaln_t_table`` (grid 1025, t_dim 8) and is
    the linear interpolation of the two rows around it, in fp32.  Its rows
    feed DiTBlocks built as the checkpoints' are: t_dim 8, apply_silu=False,
    fp16 adaLN weights (model/dit.py:655-659)."""
    grid = adaln_t_table.shape[0]
    if adaln_t_table.dim() != 2 or grid < 2:
        raise ValueError("adaln_t_table must be [grid >= 2, t_dim]")
    table = adaln_t_table.to(device=t.device, dtype=torch.float32)
    pos = t.to(torch.float32).reshape(-1).clamp(0.0, 1.0) * (grid - 1)
    lo = pos.floor().long().clamp(max=grid - 2)
    return torch.lerp(table[lo], table[lo + 1], (pos - lo).unsqueeze(1))


def quantize_linear_weight(w: torch.Tensor, fmt: str) -> dict:
    """Checkpoint-format tensors for a dense [N, K] weight (harness for random
    weights; real checkpoints arrive quantised): int8_tensorwise = symmetric
    per-output-channel INT8 + fp32 scales; nvfp4 = hi-first e2m1 codes, blocked
    e4m3 scales, fp32 per-tensor scale (the format ops/nvfp4.py decodes)."""
    if fmt == "int8_tensorwise":
        w32 = w.float()
        ws = w32.abs().amax(dim=1).clamp(min=1e-12) / 127.0
        q = (w32 / ws[:, None]).round().clamp(-128, 127).to(torch.int8)
        return {"weight": q, "weight_scale": ws, "meta": {"format": fmt}}
    if fmt == "nvfp4":
        t = ops.quant_nvfp4(w.to(torch.bfloat16).contiguous(), hi_first=True)
        return {"weight": t.codes, "weight_scale": t.sf, "weight_scale_2": t.gs, "meta": {"format": fmt}}
    raise ValueError(fmt)


def load_quant_linear(ql: QuantLinear, w: torch.Tensor, fmt: str) -> None:
    d = quantize_linear_weight(w, fmt)
    ql.set_quant(d["weight"], meta=d["meta"], weight_scale=d["weight_scale"],
                 weight_scale_2=d.get("weight_scale_2"), device=w.device)
    ql.prepare_cube()


def init_block_random(block: DiTBlock, fmt: str, gen: torch.Generator, std: float = 0.02) -> None:
    """Random N(0, std) weights for every projection of a block, quantised to
    `fmt` through the checkpoint path; norms ~1, adaLN N(0, std)."""
    dev = block.norm1.weight.device
    for ql in (block.attn.qkv_proj, block.attn.out_proj, block.mlp.fc1, block.mlp.fc2):
        w = torch.randn(ql.out_features, ql.in_features, generator=gen, device=dev) * std
        load_quant_linear(ql, w, fmt)
    lin = block.adaln_proj.linear
    lin.weight.data.copy_(torch.randn(lin.weight.shape, generator=gen, device=dev) * std)
    lin.bias.data.copy_(torch.randn(lin.bias.shape, generator=gen, device=dev) * std)
    for norm in (block.norm1, block.norm2, block.attn.q_norm, block.attn.k_norm):
        norm.weight.data.copy_(1.0 + 0.1 * torch.randn(norm.weight.shape, generator=gen, device=dev))


class DiTStep(nn.Module):
    """One denoising step of a block stack over a joint [text | video]
    sequence (the benchmark configuration): text features go through
    ``condition_proj`` (model/dit.py:668-670, 811) and are prepended to the
    video tokens; text rows use adaLN row 1, video rows row 0
    (model/dit.py:852-867).  Under Ulysses every rank holds S/ws tokens."""

    def __init__(self, *, hidden: int, heads: int, ffn: int, depth: int, text_dim: int, t_dim: int = 256,
                 fmt: str = "nvfp4", mlp_act: str = "gelu", eps: float = 1e-6, device=None,
                 seq_parallel: str = "p2p"):
        super().__init__()
        self.hidden, self.t_dim = hidden, t_dim
        self.condition_proj = QuantLinear(text_dim, hidden, bias=False, device=device)
        self.blocks = nn.ModuleList([
            DiTBlock(hidden, heads, 128, ffn, t_dim, eps, eps, apply_silu=True, dtype=torch.bfloat16,
                     device=device, mlp_act=mlp_act, seq_parallel=seq_parallel) for _ in range(depth)])
        self.fmt = fmt

    def init_random(self, seed: int = 0) -> None:
        dev = self.condition_proj.weight.device
        gen = torch.Generator(device=dev).manual_seed(seed)
        w = torch.randn(self.condition_proj.out_features, self.condition_proj.in_features, generator=gen,
                        device=dev) * 0.02
        load_quant_linear(self.condition_proj, w, self.fmt)
        for blk in self.blocks:
            init_block_random(blk, self.fmt, gen)

    def forward(self, video: torch.Tensor, text: torch.Tensor, timestep: torch.Tensor, rope: RopeSpec
                ) -> torch.Tensor:
        """video: this rank's video rows [S_local - text rows here, hidden];
        text: the full text features [n_text, text_dim] (every rank passes
        them; only ranks whose token range covers them project them).
        Returns this rank's hidden states after all blocks."""
        n_text = text.shape[0]
        s_total = rope.pos.shape[0]
        s0, s1 = split_range(s_total) if is_distributed() else (0, s_total)
        x = torch.empty((s1 - s0, self.hidden), dtype=torch.bfloat16, device=video.device)
        n_here = max(0, min(n_text, s1) - s0)
        if n_here:
            x[:n_here] = self.condition_proj(text[s0:s0 + n_here])
        x[n_here:] = video
        segments = clip_mod_segments([(0, n_text, 1), (n_text, s_total, 0)], s0, s1)
        t_emb = timestep_embedding(timestep, self.t_dim).to(torch.bfloat16)
        for blk in self.blocks:
            x = blk(x, t_emb, segments, rope)
        return x
