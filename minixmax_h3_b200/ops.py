"""Torch-facing wrappers over the C ABI (device memory, streams, shapes).

Each wrapper validates dtypes/devices, allocates its outputs with the caching
allocator, and launches on the current CUDA stream.  There is no CPU path:
non-CUDA tensors raise.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from ._lib import call

EPI_STORE, EPI_GELU, EPI_GATE_RES, EPI_SWIGLU, EPI_STORE_POSMAX = 0, 1, 2, 3, 4


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("minixmax_h3_b200 ops run on CUDA tensors only (no CPU fallback)")


def _rows(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """Views x as [m, k] with unit column stride; returns (x2, m, k, ld)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    ld = x2.stride(0) if x2.shape[0] > 1 else x2.shape[1]
    return x2, x2.shape[0], x2.shape[1], ld


# ----------------------------------------------------------------------------- INT8


def quant_i8_rows(x: torch.Tensor, *, convrot_group: int = 0,
                  x_rot_out: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row dynamic INT8 quantisation -> (q int8 [m,k], scale fp32 [m]).

    convrot_group=256 first rotates every 256-column group by the regular
    Hadamard matrix (ConvRot, ops/hadamard.py:35-44); x_rot_out, if given
    (dense [m, k], x's dtype), receives the rotated activation."""
    _cuda(x, x_rot_out)
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("quant_i8_rows expects bf16/fp16 input")
    x2, m, k, ld = _rows(x)
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    if m == 0:  # empty batch (a zero-size tensor may carry a null pointer)
        return q, s
    dt = 0 if x.dtype == torch.bfloat16 else 1
    if convrot_group:
        if x_rot_out is not None and (x_rot_out.shape != (m, k) or x_rot_out.dtype != x.dtype
                                      or not x_rot_out.is_contiguous()):
            raise ValueError("x_rot_out must be a dense [m, k] tensor of x's dtype")
        call("h3b_quant_i8_rows_convrot", x2.data_ptr(), dt, m, k, ld, int(convrot_group), q.data_ptr(),
             s.data_ptr(), x_rot_out.data_ptr() if x_rot_out is not None else None, _stream(x))
    else:
        call("h3b_quant_i8_rows", x2.data_ptr(), dt, m, k, ld, q.data_ptr(), s.data_ptr(), _stream(x))
    return q, s


def gemm_i8(q: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
            bias: Optional[torch.Tensor] = None, *, epilogue: int = EPI_STORE,
            resid: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
            row_sel: Optional[torch.Tensor] = None, amax_out: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = epi(acc * xs[m] * ws[n] + bias) in bf16; w is the [N, K] int8 weight.

    EPI_GATE_RES: y = resid + v * gate[row_sel[m]] with gate a [rows, N] table
    (a strided view is fine) and resid updated in place when out is None.
    EPI_SWIGLU: w rows interleaved by swiglu_interleave_perm; y is [m, N/2].
    """
    _cuda(q, xs, w, ws, bias, resid, gate, row_sel, amax_out, out)
    m, k = q.shape
    n = w.shape[0]
    if out is None:
        out = resid if epilogue == EPI_GATE_RES else torch.empty(
            (m, n // 2 if epilogue == EPI_SWIGLU else n), dtype=torch.bfloat16, device=q.device)
    if m == 0:
        return out
    gate_ld = _gate_ld(gate)
    call("h3b_gemm_i8_bf16", q.data_ptr(), xs.data_ptr(), w.data_ptr(), ws.data_ptr(), _ptr(bias), out.data_ptr(),
         out.stride(0), _ptr(resid), _ptr(gate), gate_ld, _ptr(row_sel), _ptr(amax_out), epilogue, m, n, k,
         _stream(q))
    return out


def gemm_i8_seq2head(q: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
                     bias: Optional[torch.Tensor], recv_ptrs: Sequence[int], rank: int, heads: int) -> None:
    """QKV GEMM whose output rows land in every head owner's receive buffer
    [ws*m, 3, heads/ws, 128] (recv_ptrs in rank order): the seq->head
    Ulysses exchange fused into the epilogue."""
    _cuda(q, xs, w, ws, bias)
    m, k = q.shape
    arr = (ctypes.c_void_p * len(recv_ptrs))(*recv_ptrs)
    call("h3b_gemm_i8_seq2head", q.data_ptr(), xs.data_ptr(), w.data_ptr(), ws.data_ptr(), _ptr(bias),
         ctypes.cast(arr, ctypes.c_void_p), len(recv_ptrs), rank, heads, m, w.shape[0], k, _stream(q))


def _gate_ld(gate: Optional[torch.Tensor]) -> int:
    if gate is None:
        return 0
    if gate.stride(-1) != 1:
        raise ValueError("gate table needs unit column stride")
    return gate.stride(0) if gate.dim() == 2 else 0


def gemm_i8_acc(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Raw int32 accumulators sum_k q[m,k]*w[n,k] from the tensor cores."""
    _cuda(q, w)
    m, k = q.shape
    n = w.shape[0]
    acc = torch.empty((m, n), dtype=torch.int32, device=q.device)
    call("h3b_gemm_i8_acc_i32", q.data_ptr(), w.data_ptr(), acc.data_ptr(), m, n, k, _stream(q))
    return acc


# ----------------------------------------------------------------------------- NVFP4


@dataclass
class NVFP4Tensor:
    """Packed NVFP4 operand: codes [rows, k/2] u8, blocked e4m3 scales, fp32 gs."""

    codes: torch.Tensor
    sf: torch.Tensor
    gs: torch.Tensor
    rows: int
    k: int
    hi_first: bool


def sf_blocked_bytes(rows: int, k: int) -> int:
    return ((rows + 127) // 128 * 128) * ((k // 16 + 3) // 4 * 4)


def amax(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _cuda(x)
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise TypeError("amax expects a contiguous bf16 tensor")
    if out is None:
        out = torch.empty((1,), dtype=torch.float32, device=x.device)
    if x.numel() == 0:
        return out.zero_()
    call("h3b_amax_bf16", x.data_ptr(), x.numel(), out.data_ptr(), _stream(x))
    return out


def quant_nvfp4(x: torch.Tensor, *, hi_first: bool = False,
                amax_t: Optional[torch.Tensor] = None) -> NVFP4Tensor:
    """Dynamic NVFP4 quantisation of a bf16 [.., k] tensor (global scale from amax)."""
    _cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("quant_nvfp4 expects bf16 input")
    x2, m, k, ld = _rows(x)
    if m == 0:  # an empty batch: no codes, and the global scale of an all-zero tensor
        return NVFP4Tensor(torch.empty((0, k // 2), dtype=torch.uint8, device=x.device),
                           torch.empty((0,), dtype=torch.uint8, device=x.device),
                           torch.ones((1,), dtype=torch.float32, device=x.device), 0, k, hi_first)
    if amax_t is None:
        amax_t = amax(x2 if x2.is_contiguous() else x2.contiguous())
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
    sf = torch.empty((sf_blocked_bytes(m, k),), dtype=torch.uint8, device=x.device)
    gs = torch.empty((1,), dtype=torch.float32, device=x.device)
    call("h3b_quant_nvfp4", x2.data_ptr(), m, k, ld, amax_t.data_ptr(), codes.data_ptr(), sf.data_ptr(),
         gs.data_ptr(), 1 if hi_first else 0, _stream(x))
    return NVFP4Tensor(codes, sf, gs, m, k, hi_first)


def gelu_amax_scan(y: torch.Tensor, ymax2: torch.Tensor) -> torch.Tensor:
    """ymax2[1] = max |bf16(gelu(y))| over fc1's bf16 output y when the bound
    from ymax2[0] = max(0, max y) does not settle max |u| (h3b_gelu_amax_scan);
    ymax2 is an fp32 [2] device tensor, ymax2[1] zero on entry."""
    _cuda(y, ymax2)
    if y.dtype != torch.bfloat16:
        raise TypeError("gelu_amax_scan expects bf16 input")
    if ymax2.dtype != torch.float32 or ymax2.numel() != 2 or not ymax2.is_contiguous():
        raise ValueError("ymax2 must be a contiguous fp32 tensor of 2 elements")
    y2, m, k, ld = _rows(y)
    call("h3b_gelu_amax_scan", y2.data_ptr(), m, k, ld, ymax2.data_ptr(), _stream(y))
    return ymax2


def quant_nvfp4_gelu(y: torch.Tensor, ymax2: torch.Tensor, *, hi_first: bool = False) -> NVFP4Tensor:
    """NVFP4 quantisation of u = bf16(gelu(y)) computed from fc1's bf16 output
    y on the fly (h3b_quant_nvfp4_gelu): the MLP activation fused with fc2's
    input quantisation.  ymax2: fp32 [2] from the fc1 GEMM's
    EPI_STORE_POSMAX max and gelu_amax_scan, max-reduced across ranks."""
    _cuda(y, ymax2)
    if y.dtype != torch.bfloat16:
        raise TypeError("quant_nvfp4_gelu expects bf16 input")
    if ymax2.dtype != torch.float32 or ymax2.numel() != 2 or not ymax2.is_contiguous():
        raise ValueError("ymax2 must be a contiguous fp32 tensor of 2 elements")
    y2, m, k, ld = _rows(y)
    if m == 0:
        raise ValueError("quant_nvfp4_gelu needs at least one row")
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=y.device)
    sf = torch.empty((sf_blocked_bytes(m, k),), dtype=torch.uint8, device=y.device)
    gs = torch.empty((1,), dtype=torch.float32, device=y.device)
    call("h3b_quant_nvfp4_gelu", y2.data_ptr(), m, k, ld, ymax2.data_ptr(), codes.data_ptr(), sf.data_ptr(),
         gs.data_ptr(), 1 if hi_first else 0, _stream(y))
    return NVFP4Tensor(codes, sf, gs, m, k, hi_first)


def swap_nibbles(u8: torch.Tensor) -> torch.Tensor:
    _cuda(u8)
    src = u8.contiguous()
    dst = torch.empty_like(src)
    call("h3b_nvfp4_swap_nibbles", src.data_ptr(), dst.data_ptr(), src.numel(), _stream(src))
    return dst


def gemm_nvfp4_seq2head(a: NVFP4Tensor, w: NVFP4Tensor, bias: Optional[torch.Tensor], recv_ptrs: Sequence[int],
                        rank: int, heads: int) -> None:
    """NVFP4 variant of gemm_i8_seq2head (both operands lo-first)."""
    if a.hi_first or w.hi_first:
        raise ValueError("gemm_nvfp4_seq2head needs tensor-core (lo-first) nibble order")
    _cuda(a.codes, w.codes, bias)
    arr = (ctypes.c_void_p * len(recv_ptrs))(*recv_ptrs)
    call("h3b_gemm_nvfp4_seq2head", a.codes.data_ptr(), a.sf.data_ptr(), a.gs.data_ptr(), w.codes.data_ptr(),
         w.sf.data_ptr(), w.gs.data_ptr(), _ptr(bias), ctypes.cast(arr, ctypes.c_void_p), len(recv_ptrs), rank,
         heads, a.rows, w.rows, a.k, _stream(a.codes))


def swiglu_interleave_perm(n: int, device=None) -> torch.Tensor:
    """Row order of an fc1 weight [n = 2*ffn, K] for EPI_SWIGLU: blocks of 32
    gate rows and the matching 32 up rows alternate, so new row 64b + j is
    gate row 32b + j and new row 64b + 32 + j is up row ffn + 32b + j
    (the halves of model/dit.py:120-129 x.chunk(2, dim=-1))."""
    if n % 64:
        raise ValueError("SwiGLU fc1 needs 2*ffn % 64 == 0")
    ffn = n // 2
    b = torch.arange(ffn // 32).repeat_interleave(32)
    j = torch.arange(32).repeat(ffn // 32)
    gate = 32 * b + j
    perm = torch.stack([gate.view(-1, 32), (ffn + gate).view(-1, 32)], dim=1).reshape(-1)
    return perm.to(device)


def _blocked_index(rows: int, ncols: int, device) -> torch.Tensor:
    """Flat offsets of every (row, scale column) of the 128x4 blocked scale
    layout (ops/nvfp4.py from_blocked), rows padded to 128: [rows_pad, ncols]."""
    rows_pad = (rows + 127) // 128 * 128
    r = torch.arange(rows_pad, device=device).view(-1, 1)
    c = torch.arange(ncols, device=device).view(1, -1)
    ncb = ncols // 4
    return ((r // 128) * ncb + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4


def permute_blocked_rows(sf: torch.Tensor, rows: int, k: int, perm: torch.Tensor) -> torch.Tensor:
    """Reorders the rows of NVFP4 block scales kept in the blocked layout
    (row i of the result = row perm[i]); padding rows stay zero."""
    ncols = k // 16
    idx = _blocked_index(rows, ncols, sf.device)
    dense = sf.reshape(-1)[idx]
    full = torch.cat([perm.to(sf.device), torch.arange(rows, idx.shape[0], device=sf.device)])
    out = torch.zeros_like(sf.reshape(-1))
    out[idx.reshape(-1)] = dense[full].reshape(-1)
    return out.view_as(sf)


def gemm_nvfp4(a: NVFP4Tensor, w: NVFP4Tensor, bias: Optional[torch.Tensor] = None, *,
               epilogue: int = EPI_STORE, resid: Optional[torch.Tensor] = None,
               gate: Optional[torch.Tensor] = None, row_sel: Optional[torch.Tensor] = None,
               amax_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = epi(a_gs*w_gs * A @ W^T + bias) in bf16; both operands lo-first."""
    if a.hi_first or w.hi_first:
        raise ValueError("gemm_nvfp4 needs tensor-core (lo-first) nibble order; repack with swap_nibbles")
    _cuda(a.codes, w.codes, bias, resid, gate, row_sel, amax_out, out)
    m, n, k = a.rows, w.rows, a.k
    if out is None:
        out = resid if epilogue == EPI_GATE_RES else torch.empty(
            (m, n // 2 if epilogue == EPI_SWIGLU else n), dtype=torch.bfloat16, device=a.codes.device)
    if m == 0:
        return out
    call("h3b_gemm_nvfp4_bf16", a.codes.data_ptr(), a.sf.data_ptr(), a.gs.data_ptr(), w.codes.data_ptr(),
         w.sf.data_ptr(), w.gs.data_ptr(), _ptr(bias), out.data_ptr(), out.stride(0), _ptr(resid), _ptr(gate),
         _gate_ld(gate), _ptr(row_sel), _ptr(amax_out), epilogue, m, n, k, _stream(a.codes))
    return out


# ----------------------------------------------------------------------------- attention


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
              out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
              amax_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Non-causal attention over token-major views q [Sq,H,128], k/v [Skv,H,128].

    Any strides with a unit last dimension are accepted (e.g. slices of a packed
    [S, 3, H, D] QKV buffer).  Returns o [Sq, H, 128] bf16.
    """
    _cuda(q, k, v, out, lse, amax_out)
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[-1] != 128 or t.stride(-1) != 1:
            raise ValueError("attention expects bf16 [S, H, 128] views with unit last stride")
    if k.stride() != v.stride():
        raise ValueError("k and v must share strides")
    s_q, heads, d = q.shape
    s_kv = k.shape[0]
    if out is None:
        out = torch.empty((s_q, heads, d), dtype=torch.bfloat16, device=q.device)
    if s_q == 0:
        return out
    scale = d ** -0.5 if scale is None else float(scale)
    call("h3b_attention_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _ptr(lse), _ptr(amax_out),
         heads, s_q,
         s_kv, q.stride(0), q.stride(1), k.stride(0), k.stride(1), out.stride(0), out.stride(1), scale, _stream(q))
    return out


def attention_merge_lse(acc: torch.Tensor, acc_lse: torch.Tensor, blk: torch.Tensor, blk_lse: torch.Tensor, *,
                        first: bool, out: Optional[torch.Tensor] = None,
                        amax_out: Optional[torch.Tensor] = None) -> None:
    """Fold one key chunk's attention result (blk bf16 [S, H, 128], blk_lse
    [H, S]) into the running fp32 result acc / acc_lse (ops/fa_h3.py:141-156);
    first=True initialises them.  With out (bf16 [S, H, 128]) given, the merged
    rows go there (and max |out| into amax_out) instead of acc."""
    _cuda(acc, acc_lse, blk, blk_lse, out, amax_out)
    s, heads, d = blk.shape
    if d != 128 or acc.shape != blk.shape or acc_lse.shape != (heads, s) or blk_lse.shape != (heads, s):
        raise ValueError("attention_merge_lse: acc/blk [S, H, 128], lse [H, S]")
    if acc.dtype != torch.float32 or blk.dtype != torch.bfloat16 or acc_lse.dtype != torch.float32 \
            or blk_lse.dtype != torch.float32:
        raise ValueError("attention_merge_lse: acc fp32, blk bf16, lse fp32")
    tensors = (acc, acc_lse, blk, blk_lse) + ((out,) if out is not None else ())
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("attention_merge_lse: contiguous tensors only")
    if out is not None and (out.shape != blk.shape or out.dtype != torch.bfloat16):
        raise ValueError("attention_merge_lse: out bf16 [S, H, 128]")
    call("h3b_attention_merge_lse", acc.data_ptr(), acc_lse.data_ptr(), blk.data_ptr(), blk_lse.data_ptr(), s, heads,
         1 if first else 0, _ptr(out), _ptr(amax_out), _stream(blk))


def attention_head2seq(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o_ptrs: Sequence[int], *,
                       s_local: int, head0: int, total_heads: int, scale: Optional[float] = None,
                       amax_out: Optional[torch.Tensor] = None) -> None:
    """Attention over this rank's heads (q/k/v [S, H_local, 128] views of all
    S tokens) writing query row t into rank t // s_local's out-projection
    input [s_local, total_heads, 128] (o_ptrs[r]: device pointers valid in
    this process, rank order) at head head0 + h — the head->sequence Ulysses
    exchange fused into the epilogue."""
    _cuda(q, k, v, amax_out)
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[-1] != 128 or t.stride(-1) != 1:
            raise ValueError("attention expects bf16 [S, H, 128] views with unit last stride")
    if k.stride() != v.stride():
        raise ValueError("k and v must share strides")
    s_q, heads, d = q.shape
    scale = d ** -0.5 if scale is None else float(scale)
    arr = (ctypes.c_void_p * len(o_ptrs))(*o_ptrs)
    call("h3b_attention_fwd_head2seq", q.data_ptr(), k.data_ptr(), v.data_ptr(), ctypes.cast(arr, ctypes.c_void_p),
         len(o_ptrs), s_local, head0, total_heads * d, d, _ptr(amax_out), heads, s_q, k.shape[0], q.stride(0),
         q.stride(1), k.stride(0), k.stride(1), scale, _stream(q))


def qk_rmsnorm_rope(q: torch.Tensor, k: Optional[torch.Tensor], q_weight: torch.Tensor,
                    k_weight: Optional[torch.Tensor], eps: float, pos: torch.Tensor, pos_offset: int,
                    inv_freq: torch.Tensor, n_t: int, n_h: int) -> None:
    """In-place RMSNorm + split-half RoPE of q (and k) [S, H, 128] views."""
    _cuda(q, k, q_weight, k_weight, pos, inv_freq)
    if k is not None and k.stride() != q.stride():
        raise ValueError("q and k must share strides")
    s, heads, d = q.shape
    call("h3b_qk_rmsnorm_rope", q.data_ptr(), _ptr(k), s, heads, q.stride(0), q.stride(1), q_weight.data_ptr(),
         _ptr(k_weight), eps, pos.data_ptr(), pos_offset, inv_freq.data_ptr(), n_t, n_h, _stream(q))


# ----------------------------------------------------------------------------- block elementwise


def rmsnorm_modulate(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float,
                     row_sel: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                     amax_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """h = rmsnorm(x)*w*(1+scale[row_sel]) + shift[row_sel]; shift/scale are
    [rows, hidden] tables (strided views of the adaLN output are fine)."""
    _cuda(x, weight, shift, scale, row_sel, out, amax_out)
    x2, m, hidden, ld = _rows(x)
    if out is None:
        out = torch.empty((m, hidden), dtype=torch.bfloat16, device=x.device)
    if shift.stride() != scale.stride():
        raise ValueError("shift and scale tables must share strides")
    if out.stride(0) != ld:
        raise ValueError("out must share the row stride of x")
    call("h3b_rmsnorm_modulate", x2.data_ptr(), out.data_ptr(), m, hidden, ld, weight.data_ptr(), shift.data_ptr(),
         scale.data_ptr(), _gate_ld(shift), _ptr(row_sel), eps, _ptr(amax_out), _stream(x))
    return out


def rmsnorm_modulate_quant_i8(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                              eps: float, row_sel: Optional[torch.Tensor] = None, convrot_group: int = 0,
                              q_out: Optional[torch.Tensor] = None, scale_out: Optional[torch.Tensor] = None
                              ) -> tuple[torch.Tensor, torch.Tensor]:
    """rmsnorm_modulate(x, ...) followed by quant_i8_rows(h, convrot_group)
    in one kernel (h is never written): returns (q [m, hidden] int8,
    per-row scale [m] fp32), the same bits as the two calls."""
    _cuda(x, weight, shift, scale, row_sel, q_out, scale_out)
    x2, m, hidden, ld = _rows(x)
    if shift.stride() != scale.stride():
        raise ValueError("shift and scale tables must share strides")
    if convrot_group not in (0, 256):
        raise NotImplementedError(f"ConvRot group size {convrot_group}: this build rotates 256-column groups")
    q = q_out if q_out is not None else torch.empty((m, hidden), dtype=torch.int8, device=x.device)
    xs = scale_out if scale_out is not None else torch.empty(m, dtype=torch.float32, device=x.device)
    if q.shape != (m, hidden) or not q.is_contiguous() or xs.numel() != m:
        raise ValueError("rmsnorm_modulate_quant_i8: q [m, hidden] contiguous, scale [m]")
    call("h3b_rmsnorm_modulate_quant_i8", x2.data_ptr(), m, hidden, ld, weight.data_ptr(), shift.data_ptr(),
         scale.data_ptr(), _gate_ld(shift), _ptr(row_sel), eps, convrot_group, q.data_ptr(), xs.data_ptr(),
         _stream(x))
    return q, xs


def gate_residual(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor,
                  row_sel: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x += y * gate[row_sel] in place (bf16)."""
    _cuda(x, y, gate, row_sel)
    m, hidden = x.shape
    if y.stride() != x.stride():
        raise ValueError("x and y must share strides")
    call("h3b_gate_residual", x.data_ptr(), y.data_ptr(), m, hidden, x.stride(0), gate.data_ptr(), _gate_ld(gate),
         _ptr(row_sel), _stream(x))
    return x


# ----------------------------------------------------------------------------- reference-named entries


def rotate_activation(x: torch.Tensor, group_size: int) -> torch.Tensor:
    """ops/hadamard.py:35-44: x [..., K] times the regular Hadamard matrix in
    every group_size-column group (ConvRot's online rotation).  This build
    rotates 256-column groups, exactly in fp64 and rounded once to x's dtype;
    the reference's value comes from a 16-bit GEMM, which can differ from the
    exact one by a unit in the last place.  Runs the rotating quantiser and
    keeps its rotated rows."""
    if group_size != 256:
        raise NotImplementedError(f"ConvRot group size {group_size}: this build rotates 256-column groups")
    *lead, k = x.shape
    if k % group_size != 0:
        raise ValueError(f"K={k} not divisible by group_size={group_size}")
    x2 = x.reshape(-1, k)
    out = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    quant_i8_rows(x2, convrot_group=group_size, x_rot_out=out)
    return out.reshape(*lead, k)


def int8_convrot_linear(x: torch.Tensor, weight_i8: torch.Tensor, weight_scale: torch.Tensor,
                        bias: Optional[torch.Tensor] = None, *, convrot: bool = True, group_size: int = 256,
                        out_dtype: torch.dtype = torch.bfloat16, weight_layout: str = "nk") -> torch.Tensor:
    """ops/int8_convrot.py:114-209: y = W8A8(x) with x [..., K] cast to
    out_dtype, optionally ConvRot-rotated, quantised per row and multiplied
    by the [N, K] int8 weight with its per-channel scales (+ bias).

    The ``nk`` layout is the only one: the reference's ``kn`` / ``nz29`` are
    its NPU Cube packings.  The output is bf16 (the GEMM's epilogue rounds
    once to bf16; an fp16 result would round twice), so other out_dtypes are
    refused rather than approximated.  Non-CUDA tensors raise RuntimeError,
    as the reference does for non-NPU ones."""
    if weight_layout != "nk":
        raise ValueError(f"weight_layout {weight_layout!r}: the tcgen05 GEMM reads the [N, K] int8 weight as stored")
    if out_dtype != torch.bfloat16:
        raise NotImplementedError(f"out_dtype {out_dtype}: the INT8 GEMM writes bf16")
    *lead, k = x.shape
    x2 = x.reshape(-1, k).to(out_dtype)
    q, xs = quant_i8_rows(x2, convrot_group=group_size if convrot else 0)
    b = bias.to(device=x.device, dtype=torch.bfloat16) if bias is not None else None
    y = gemm_i8(q, xs, weight_i8, weight_scale.reshape(-1).to(device=x.device, dtype=torch.float32), b)
    return y.reshape(*lead, weight_i8.shape[0])
