"""CPU oracle for the MiniMax-H3 DiT-block hot path — TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the reference algorithm of every function on
the hot path, so that tests/, ``__graft_entry__.smoke()`` and the CPU leg of
``bench.py`` can check (never replace) the CUDA kernels.  The product package
must never import it.  Reference paths are relative to
``Ref2VA-910C-FastAPI-INT8-CANN9.1.0/runtime/src/h3_npu/`` of BHUHD/minixmax-h3.

Parity pins (tests/test_oracle_pins.py, tests/golden/):
  * INT8 row quantiser, RMSNorm, RoPE table/apply, SDPA attention, Ulysses
    permutations, NVFP4 decode and the DiT block structure are checked
    bit-for-bit against the reference's own Python run in this container, and
    frozen as golden fixtures under tests/golden/ (generator committed).
  * The W8A8 int32 GEMM and the NVFP4 *quantiser* have no CPU implementation
    in the reference (vendor kernels / the unvendored comfy_kitchen package):
    they are restated here from their published semantics, and the NVFP4
    quantiser is pinned only through the reference decode round trip
    (``dequantize_nvfp4(quantize(x))``) — parity of the quantiser itself is
    unpinned.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import numpy as np
import torch
import torch.nn.functional as F

# ----------------------------------------------------------------------------- INT8 W8A8


def dynamic_quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row dynamic INT8 (ops/int8_convrot.py:107-111, the host path).

    amax = max|x| per row clamped to 1e-12; scale = amax/127 (fp32);
    q = round_half_even(x/scale) clamped to [-128, 127].
    """
    x2 = x.float()
    amax = x2.abs().amax(dim=-1).clamp(min=1e-12)
    scale = amax / 127.0
    q = (x2 / scale.unsqueeze(-1)).round().clamp(-128, 127).to(torch.int8)
    return q, scale


H4 = ((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1))


def hadamard_matrix(size: int) -> np.ndarray:
    """Regular Hadamard H4 (x) ... (x) H4 / sqrt(size) in fp64
    (ops/hadamard.py:11-32: kron powers of the H4 seed, size a power of 4)."""
    if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
        raise ValueError("size must be a power of 4")
    h4 = np.array(H4, dtype=np.float64)
    h = h4
    while h.shape[0] < size:
        h = np.kron(h, h4)
    return h / np.sqrt(size)


def round_f64_to_16(v: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """One round-to-nearest-even from fp64 to bf16 / fp16 (no intermediate
    fp32 rounding).  bf16: the fp64 significand is rounded at bit 45 (keeping
    8 significant bits), exact for results in the bf16 normal range; fp16:
    numpy's direct double->half conversion."""
    v = np.ascontiguousarray(v, dtype=np.float64)
    if dtype == torch.float16:
        return torch.from_numpy(v.astype(np.float16))
    if dtype != torch.bfloat16:
        raise TypeError(dtype)
    u = v.view(np.uint64)
    keep = (u >> np.uint64(45)) & np.uint64(1)
    r = (u + np.uint64((1 << 44) - 1) + keep) & ~np.uint64((1 << 45) - 1)
    f32 = r.view(np.float64).astype(np.float32)  # exact: 8 significant bits
    return torch.from_numpy(f32).to(torch.bfloat16)  # exact truncation


def rotate_activation_exact(x: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """ConvRot online rotation (ops/hadamard.py:35-44): every group of
    `group_size` columns times the regular Hadamard matrix, in x's 16-bit
    dtype.  Restated as the exact product (fp64 holds every partial sum of
    16-bit inputs with +-1 coefficients exactly for groups whose magnitudes
    span under 2^37) rounded once to the output dtype; the reference's value
    comes from a 16-bit GEMM with backend-defined fp32 accumulation order."""
    *lead, k = x.shape
    if k % group_size:
        raise ValueError("k must be a multiple of group_size")
    h = hadamard_matrix(group_size)
    xd = x.reshape(-1, group_size).to(torch.float64).numpy()
    y = xd @ h
    return round_f64_to_16(y, x.dtype).reshape(*lead, k)


def quantize_weight_int8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel INT8 weights (harness; the reference ships
    pre-quantised checkpoints, load/safetensors_quant.py:65-78)."""
    w32 = w.float()
    ws = w32.abs().amax(dim=1).clamp(min=1e-12) / 127.0
    q = (w32 / ws.unsqueeze(1)).round().clamp(-128, 127).to(torch.int8)
    return q, ws


def int8_acc(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Exact int32 accumulators sum_k q[m,k]*w[n,k] (fp64 matmul is exact here:
    |acc| <= k*128*128 < 2**53)."""
    acc = q.to(torch.float64) @ w.to(torch.float64).T
    return acc.to(torch.int64).to(torch.int32)


def w8a8_linear(q: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
                bias: Optional[torch.Tensor] = None, acc: Optional[torch.Tensor] = None) -> torch.Tensor:
    """npu_quant_matmul semantics (ops/int8_convrot.py:86-93): acc*xs[m]*ws[n]
    (+bias) in fp32, then bf16."""
    if acc is None:
        acc = int8_acc(q, w)
    y = acc.float() * xs.float()[:, None] * ws.float()[None, :]
    if bias is not None:
        y = y + bias.float()
    return y.to(torch.bfloat16)


# ----------------------------------------------------------------------------- NVFP4

# e2m1 value of each 4-bit code (ops/nvfp4.py:22-39).
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    """OCP e4m3fn byte -> fp32 (ops/float8_cast.py:21-34): bias 7, subnormals
    mant/8 * 2^-6, 0x7F/0xFF NaN."""
    b = bits.astype(np.int32)
    sign = (b >> 7) & 1
    exp = (b >> 3) & 0xF
    mant = b & 0x7
    val = np.where(exp == 0, mant.astype(np.float32) / 8.0 * np.float32(2.0 ** -6),
                   (1.0 + mant.astype(np.float32) / 8.0) * np.exp2((exp - 7).astype(np.float32)))
    val = np.where((exp == 15) & (mant == 7), np.float32(np.nan), val).astype(np.float32)
    return np.where(sign == 1, -val, val).astype(np.float32)


_E4M3_POS = e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8))  # 0x00..0x7E ascending, 0..448


def e4m3_rn_satfinite(v: np.ndarray) -> np.ndarray:
    """Non-negative fp32 -> e4m3fn byte, round-to-nearest-even, saturating at 448."""
    v = np.asarray(v, dtype=np.float32)
    if np.any(v < 0) or np.any(np.isnan(v)):
        raise ValueError("e4m3_rn_satfinite expects finite non-negative inputs")
    n = len(_E4M3_POS)
    idx = np.searchsorted(_E4M3_POS, v, side="left")  # first code whose value >= v
    hi = np.minimum(idx, n - 1)
    lo = np.maximum(hi - 1, 0)
    d_hi = _E4M3_POS[hi].astype(np.float64) - v.astype(np.float64)
    d_lo = v.astype(np.float64) - _E4M3_POS[lo].astype(np.float64)
    # even code == even mantissa (the mantissa is the low 3 bits)
    pick_hi = (d_hi == 0) | (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(idx == 0, 0, code)
    code = np.where(v >= _E4M3_POS[-1], n - 1, code)
    return code.astype(np.uint8)


def e2m1_rne_sat(r: np.ndarray) -> np.ndarray:
    """fp32 -> 4-bit e2m1 code, round-half-even on |r|, saturating at 6; sign
    bit taken from the fp32 sign (so -0.1 -> code 8)."""
    a = np.abs(r)
    mag = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return (mag | (np.signbit(r).astype(np.uint8) << 3)).astype(np.uint8)


def blocked_offset(rows: np.ndarray, cols: np.ndarray, ncols: int) -> np.ndarray:
    """Byte offset of scale (r, c) in the 128x4 blocked layout that
    ops/nvfp4.py:46-62 (from_blocked) un-swizzles."""
    ncb = (ncols + 3) // 4
    return (((rows // 128) * ncb + cols // 4) * 512 + (rows % 32) * 16 + ((rows % 128) // 32) * 4 + cols % 4)


def to_blocked(sf: np.ndarray) -> np.ndarray:
    """Logical [rows, ncols] scale bytes -> flat padded blocked layout."""
    rows, ncols = sf.shape
    out = np.zeros(((rows + 127) // 128 * 128) * ((ncols + 3) // 4 * 4), dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(ncols), indexing="ij")
    out[blocked_offset(r, c, ncols)] = sf
    return out


def from_blocked(flat: np.ndarray, rows: int, ncols: int) -> np.ndarray:
    r, c = np.meshgrid(np.arange(rows), np.arange(ncols), indexing="ij")
    return flat[blocked_offset(r, c, ncols)]


def nvfp4_quantize(x: torch.Tensor, hi_first: bool = True, amax: Optional[float] = None) -> dict:
    """NVFP4 quantiser restated from the published recipe (e2m1 values, one
    e4m3 scale per 16 elements, fp32 global scale):

        gs   = amax(|x|) / (6*448)   (1 when amax == 0)
        s_b  = e4m3_rn_satfinite(amax_b / (6*gs))
        code = e2m1_rne_sat(x / (s_b*gs))      (0 when s_b == 0)

    Codes are packed two per byte (hi_first: even element in the high nibble,
    the order ops/nvfp4.py:113-121 decodes); scales in the blocked layout.
    `amax` overrides max|x| for rows sampled from a larger tensor, whose
    global scale comes from the whole tensor.
    """
    xf = x.float().numpy().astype(np.float32)
    m, k = xf.shape
    if k % 16:
        raise ValueError("k must be a multiple of 16")
    if amax is not None:
        amax = np.float32(amax)
    else:
        amax = np.float32(np.abs(xf).max()) if xf.size else np.float32(0)
    gs = np.float32(amax / np.float32(2688.0)) if amax > 0 else np.float32(1.0)
    six_gs = np.float32(np.float32(6.0) * gs)
    blocks = xf.reshape(m, k // 16, 16)
    amax_b = np.abs(blocks).max(axis=-1).astype(np.float32)
    s_bits = e4m3_rn_satfinite((amax_b / six_gs).astype(np.float32))
    s_val = e4m3_decode(s_bits)
    denom = (s_val * gs).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = (blocks / denom[..., None]).astype(np.float32)
    codes = e2m1_rne_sat(r)
    codes = np.where((s_val > 0)[..., None], codes, 0).astype(np.uint8).reshape(m, k)
    even, odd = codes[:, 0::2], codes[:, 1::2]
    packed = ((even << 4) | odd) if hi_first else ((odd << 4) | even)
    return {
        "codes": torch.from_numpy(packed.astype(np.uint8)),
        "sf_logical": torch.from_numpy(s_bits),
        "sf": torch.from_numpy(to_blocked(s_bits)),
        "gs": torch.tensor([gs], dtype=torch.float32),
        "amax": float(amax),
    }


def nvfp4_dequantize(codes: torch.Tensor, gs: torch.Tensor, sf_flat: torch.Tensor, k: int,
                     hi_first: bool = True) -> torch.Tensor:
    """Exact fp32 decode (ops/nvfp4.py:86-110 without the final bf16 cast)."""
    c = codes.numpy()
    hi, lo = (c >> 4) & 0xF, c & 0xF
    idx = np.stack([hi, lo] if hi_first else [lo, hi], axis=-1).reshape(c.shape[0], -1)
    vals = E2M1_VALUES[idx]
    rows = c.shape[0]
    s = e4m3_decode(from_blocked(sf_flat.numpy(), rows, k // 16))
    out = vals.reshape(rows, k // 16, 16) * (np.float32(gs.reshape(-1)[0].item()) * s)[..., None]
    return torch.from_numpy(out.reshape(rows, k).astype(np.float32))


def nvfp4_linear_w4a4(a: dict, w: dict, k: int, bias: Optional[torch.Tensor] = None,
                      a_hi_first: bool = True, w_hi_first: bool = True) -> torch.Tensor:
    """fp64 product of the exactly decoded operands (+bias), in fp32."""
    ad = nvfp4_dequantize(a["codes"], a["gs"], a["sf"], k, a_hi_first).double()
    wd = nvfp4_dequantize(w["codes"], w["gs"], w["sf"], k, w_hi_first).double()
    y = ad @ wd.T
    if bias is not None:
        y = y + bias.double()
    return y.float()


def swap_nibbles(u8: torch.Tensor) -> torch.Tensor:
    return ((u8 >> 4) | (u8 << 4)).to(torch.uint8)


# ----------------------------------------------------------------------------- norm / RoPE


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """modules/linear.py:29-32, ops/rope.py:24-27: fp32 math, cast back."""
    orig = x.dtype
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return (x32 * weight.float()).to(orig)


def rope_inv_freq(dims: Sequence[int] = (44, 42, 42), theta: float = 10000.0) -> torch.Tensor:
    """Per-axis inverse frequencies 10000^(-2i/d), i < d/2, concatenated t|h|w."""
    parts = [1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d)) for d in dims]
    return torch.cat(parts)


def rope_angles(pos: torch.Tensor, inv_freq: torch.Tensor, n_t: int, n_h: int) -> torch.Tensor:
    """model/dit.py:746-752 (rope_freqs): per-axis pos*inv, cat(t,h,w), then
    cat(half, half).  pos: [S, 3] fp32."""
    pos = pos.to(torch.float32)
    inv = inv_freq.to(torch.float32)
    t_f = pos[:, 0:1] * inv[:n_t]
    h_f = pos[:, 1:2] * inv[n_t:n_t + n_h]
    w_f = pos[:, 2:3] * inv[n_t + n_h:]
    half = torch.cat((t_f, h_f, w_f), dim=-1)
    return torch.cat((half, half), dim=-1)


def rope_rotation_table(angles: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """ops/rope.py:7-13: [S, rot] -> [1, S, 1, rot/2, 2, 2] of [[c,-s],[s,c]]."""
    half = angles.shape[-1] // 2
    ang = angles[:, :half]
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([c, -s, s, c], dim=-1).reshape(1, angles.shape[0], 1, half, 2, 2).to(dtype)


def apply_rope_split_half(x: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """ops/rope.py:30-38: pair element j with j+D/2, arithmetic in table dtype."""
    t_ = x.reshape(*x.shape[:-1], 2, -1).movedim(-2, -1).unsqueeze(-2).to(dtype=table.dtype)
    t_out = table[..., 0] * t_[..., 0] + table[..., 1] * t_[..., 1]
    return t_out.movedim(-1, -2).reshape(*x.shape).type_as(x)


def rms_rope_apply(x: torch.Tensor, table: torch.Tensor, weight: torch.Tensor, eps: float,
                   rot_dim: int) -> torch.Tensor:
    """ops/rope.py:41-55.  x: [1, S, H, D]."""
    x = rms_norm(x, weight, eps)
    if rot_dim and rot_dim != x.shape[-1]:
        return torch.cat([apply_rope_split_half(x[..., :rot_dim], table), x[..., rot_dim:]], dim=-1)
    return apply_rope_split_half(x, table)


def grid_positions(t: int, h: int, w: int) -> torch.Tensor:
    """Integer (t, h, w) positions of a t*h*w latent grid, row-major, fp32 [S,3]."""
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    return torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], dim=-1).to(torch.float32)


# ----------------------------------------------------------------------------- attention


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None
                   ) -> torch.Tensor:
    """Non-causal softmax(q k^T * scale) v in fp32 — the SDPA host path of
    ops/attention.py:115-117 and ops/fa_h3.py:241-245.  q/k/v: [H, S, D]."""
    d = q.shape[-1]
    scale = d ** -0.5 if scale is None else scale
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=scale)


def attention_lse_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """(o, lse) of non-causal attention in fp32, token-major q [Sq, H, D],
    k/v [Skv, H, D]: o [Sq, H, D] and the natural-log row log-sum-exp
    [H, Sq] — what the FA call with softmax_lse_flag returns in
    ops/fa_h3.py:207-210."""
    d = q.shape[-1]
    scale = d ** -0.5 if scale is None else scale
    logits = torch.einsum("shd,thd->hst", q.float(), k.float()) * scale
    lse = torch.logsumexp(logits, dim=-1)
    o = torch.einsum("hst,thd->shd", torch.softmax(logits, dim=-1), v.float())
    return o, lse


def merge_lse(acc_o: torch.Tensor, acc_lse: torch.Tensor, blk_o: torch.Tensor, blk_lse: torch.Tensor
              ) -> tuple[torch.Tensor, torch.Tensor]:
    """ops/fa_h3.py:141-156 (_merge_lse) for token-major o [S, H, D] and
    lse [H, S]: o - sigmoid(l_b - l_o) * (o - o_b), l_o - logsigmoid(l_o - l_b),
    in fp32."""
    o, bo = acc_o.float(), blk_o.float()
    lo, ln = acc_lse.float().t()[..., None], blk_lse.float().t()[..., None]  # [S, H, 1]
    o = o - torch.sigmoid(ln - lo) * (o - bo)
    lo = lo - F.logsigmoid(lo - ln)
    return o, lo[..., 0].t().contiguous()


# ----------------------------------------------------------------------------- Ulysses


def seq_to_head_local(x_full: torch.Tensor, ws: int, rank: int) -> torch.Tensor:
    """What rank `rank` holds after all_to_all_heads(gather_seq=True)
    (ops/ulysses.py:23-31): all S tokens, heads [rank*H/ws, (rank+1)*H/ws)."""
    s, h, d = x_full.shape
    hl = h // ws
    return x_full[:, rank * hl:(rank + 1) * hl, :].contiguous()


def split_range(seq_len: int, ws: int, rank: int) -> tuple[int, int]:
    """ops/ulysses.py:44-50."""
    if seq_len % ws:
        raise RuntimeError(f"seq_len={seq_len} not divisible by world_size={ws} (pad tokens)")
    c = seq_len // ws
    return rank * c, (rank + 1) * c


def clip_mod_segments(segments, s0: int, s1: int):
    """ops/ulysses.py:53-61."""
    out = []
    for a, b, row in segments:
        aa, bb = max(a, s0), min(b, s1)
        if aa < bb:
            out.append((aa - s0, bb - s0, row))
    return out


# ----------------------------------------------------------------------------- DiT block


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    """[cos(t*f), sin(t*f)], f_i = max_period^(-i/(dim/2)): the 256-d
    sinusoidal embedding of the benchmark configuration."""
    half = dim // 2
    f = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32) / half)
    a = t.float()[:, None] * f[None]
    return torch.cat([torch.cos(a), torch.sin(a)], dim=-1)


def mod_scale_shift(h: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, segments) -> torch.Tensor:
    """model/dit.py:332-335 (in place, activation dtype)."""
    for a, b, row in segments:
        h[a:b].mul_(1.0 + scale[row].to(h.dtype)).add_(shift[row].to(h.dtype))
    return h


def mod_gate(x: torch.Tensor, gate: torch.Tensor, other: torch.Tensor, segments) -> torch.Tensor:
    """model/dit.py:338-341 (in place)."""
    for a, b, row in segments:
        x[a:b].addcmul_(other[a:b], gate[row].to(x.dtype))
    return x


class EmulatedQuantLinear(torch.nn.Module):
    """Quantised linear evaluated on the CPU: the operand quantisation of the
    CUDA path, dequantised exactly, product in fp64, output bf16."""

    def __init__(self, weight: torch.Tensor, fmt: str, bias: Optional[torch.Tensor] = None,
                 convrot: bool = False):
        super().__init__()
        self.fmt = fmt
        self.convrot = convrot
        self.bias = bias
        self.out_features, self.in_features = weight.shape
        if fmt == "int8":
            self.wq, self.ws = quantize_weight_int8(weight)
        elif fmt == "nvfp4":
            self.w = nvfp4_quantize(weight.to(torch.bfloat16), hi_first=True)
        else:
            raise ValueError(fmt)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16)
        if self.fmt == "int8":
            if self.convrot:  # ops/int8_convrot.py:139-140: rotate, then quantise
                x2 = rotate_activation_exact(x2, 256)
            q, xs = dynamic_quant_rows(x2)
            y = w8a8_linear(q, xs, self.wq, self.ws, self.bias)
        else:
            a = nvfp4_quantize(x2, hi_first=True)
            y = nvfp4_linear_w4a4(a, self.w, self.in_features, self.bias).to(torch.bfloat16)
        return y.reshape(*lead, self.out_features)


def dit_block_forward(x: torch.Tensor, t_emb: torch.Tensor, segments, params: dict, *, heads: int,
                      head_dim: int, eps: float, qk_eps: float, mlp_act: str, pos: torch.Tensor,
                      inv_freq: torch.Tensor, n_t: int, n_h: int, linear, attn_fp32: bool = True
                      ) -> torch.Tensor:
    """One DiT block (model/dit.py:400-438 with Attention 156-289, MLP
    291-301, AdalnProj 304-329), single rank.  `linear(name, x)` evaluates the
    block's projections; mlp_act is "gelu" (benchmark shape) or "swiglu"
    (the reference's MLP).  x: [S, hidden] bf16 (updated in place, as the
    reference does).  attn_fp32=False evaluates attention exactly as the
    reference's host path does (bf16 SDPA on [1, H, S, D]) for bit-exact pins;
    True evaluates it in fp32 (the accuracy target for the CUDA kernel)."""
    s_len, hidden = x.shape
    te = F.silu(t_emb) if params.get("adaln_silu", True) else t_emb
    ada = F.linear(te, params["adaln_w"].to(te.dtype), params["adaln_b"].to(te.dtype))
    ada = ada.view(ada.shape[0] * 3, 6 * hidden).chunk(6, dim=-1)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = ada
    h = mod_scale_shift(rms_norm(x, params["norm1_w"], eps), shift_msa, scale_msa, segments)
    qkv = linear("qkv", h)
    q, k, v = qkv.split(heads * head_dim, dim=-1)
    q = q.reshape(s_len, heads, head_dim)
    k = k.reshape(s_len, heads, head_dim)
    v = v.reshape(s_len, heads, head_dim)
    table = rope_rotation_table(rope_angles(pos, inv_freq, n_t, n_h), x.dtype)
    q = rms_rope_apply(q.unsqueeze(0), table, params["q_norm_w"], qk_eps, head_dim)[0]
    k = rms_rope_apply(k.unsqueeze(0), table, params["k_norm_w"], qk_eps, head_dim)[0]
    qb, kb, vb = (t.permute(1, 0, 2).contiguous() for t in (q, k, v))
    if attn_fp32:
        o = attention_fp32(qb, kb, vb).to(x.dtype)
    else:
        o = F.scaled_dot_product_attention(qb[None], kb[None], vb[None], scale=head_dim ** -0.5)[0]
    o = o.permute(1, 0, 2).reshape(s_len, heads * head_dim)
    x = mod_gate(x, gate_msa, linear("out", o), segments)
    h = mod_scale_shift(rms_norm(x, params["norm2_w"], eps), shift_mlp, scale_mlp, segments)
    u = linear("fc1", h)
    if mlp_act == "gelu":
        u = F.gelu(u)
    else:
        gate_, up = u.chunk(2, dim=-1)
        u = F.silu(gate_) * up
    return mod_gate(x, gate_mlp, linear("fc2", u), segments)
