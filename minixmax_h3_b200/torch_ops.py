"""``torch.ops.h3b.*``: the hot path's kernels as torch custom operators.

The reference registers its gathered attention as a custom operator
(``torch.library.custom_op("h3::gather_fa_bnsd", mutates_args=())`` with a
``register_fake``, ops/gather_fa.py:195-206) so that it composes with torch's
tracing.  Importing this module registers the same kind of operator for each
kernel of the path:

    h3b::quant_i8_rows(x, convrot_group) -> (q int8 [m, k], scale fp32 [m])
    h3b::gemm_i8(q, xs, w, ws, bias, epilogue) -> y bf16 [m, n] ([m, n/2] SwiGLU)
    h3b::quant_nvfp4(x, hi_first) -> (codes u8 [m, k/2], blocked scales u8, gs fp32 [1])
    h3b::gelu_amax_scan(y, ymax2) -> None  (updates ymax2[1]; see ops.gelu_amax_scan)
    h3b::quant_nvfp4_gelu(y, ymax2, hi_first) -> (codes, blocked scales, gs) of bf16(gelu(y))
    h3b::gemm_nvfp4(a_codes, a_sf, a_gs, w_codes, w_sf, w_gs, bias, epilogue) -> y bf16
    h3b::attention(q, k, v, scale) -> o bf16 [S, H, 128]          (token-major)
    h3b::attention_bnsd(q, k, v, scale) -> o bf16 [1, H, S, 128]  (h3_attention_bnsd)
    h3b::rmsnorm_modulate(x, weight, shift, scale, eps, row_sel) -> h bf16 [m, hidden]
    h3b::rmsnorm_modulate_quant_i8(x, weight, shift, scale, eps, row_sel, convrot_group)
        -> (q int8 [m, hidden], scale fp32 [m])

Each is registered for CUDA tensors only, so tensors on any other device raise
(there is no CPU fallback).  Each forwards to the ``ops`` function of the same
name, where a failing status code becomes a RuntimeError.  Each has a fake
implementation giving the output shapes and dtypes without running anything.
The operators write only fresh outputs (``mutates_args=()``; gelu_amax_scan
declares the one fp32 pair it updates), so the epilogue
that updates a residual in place (EPI_GATE_RES) is refused here; the modules
use it through ``ops`` directly.  NVFP4 operands are in the tensor cores'
nibble order (``ops.quant_nvfp4(hi_first=False)``, ``QuantLinear.prepare_cube``).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .attention import h3_attention_bnsd

_GEMM_EPILOGUES = (ops.EPI_STORE, ops.EPI_GELU, ops.EPI_SWIGLU)


def _rows_of(x: torch.Tensor) -> int:
    n = 1
    for d in x.shape[:-1]:
        n *= d
    return n


def _gemm_cols(n: int, epilogue: int) -> int:
    if epilogue not in _GEMM_EPILOGUES:
        raise ValueError(f"epilogue {epilogue}: the operator offers EPI_STORE, EPI_GELU and EPI_SWIGLU "
                         "(EPI_GATE_RES updates its residual in place; use ops.gemm_* for it)")
    return n // 2 if epilogue == ops.EPI_SWIGLU else n


# ----------------------------------------------------------------------------- implementations


def _quant_i8_rows(x: torch.Tensor, convrot_group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.quant_i8_rows(x, convrot_group=convrot_group)


def _gemm_i8(q: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
             bias: Optional[torch.Tensor] = None, epilogue: int = 0) -> torch.Tensor:
    _gemm_cols(w.shape[0], epilogue)
    return ops.gemm_i8(q, xs, w, ws, bias, epilogue=epilogue)


def _quant_nvfp4(x: torch.Tensor, hi_first: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    t = ops.quant_nvfp4(x, hi_first=hi_first)
    return t.codes, t.sf, t.gs


def _gelu_amax_scan(y: torch.Tensor, ymax2: torch.Tensor) -> None:
    ops.gelu_amax_scan(y, ymax2)


def _quant_nvfp4_gelu(y: torch.Tensor, ymax2: torch.Tensor,
                      hi_first: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    t = ops.quant_nvfp4_gelu(y, ymax2, hi_first=hi_first)
    return t.codes, t.sf, t.gs


def _gemm_nvfp4(a_codes: torch.Tensor, a_sf: torch.Tensor, a_gs: torch.Tensor, w_codes: torch.Tensor,
                w_sf: torch.Tensor, w_gs: torch.Tensor, bias: Optional[torch.Tensor] = None,
                epilogue: int = 0) -> torch.Tensor:
    _gemm_cols(w_codes.shape[0], epilogue)
    k = 2 * a_codes.shape[1]
    if w_codes.shape[1] * 2 != k:
        raise ValueError(f"gemm_nvfp4: activation K {k} vs weight K {w_codes.shape[1] * 2}")
    a = ops.NVFP4Tensor(a_codes, a_sf, a_gs, a_codes.shape[0], k, False)
    w = ops.NVFP4Tensor(w_codes, w_sf, w_gs, w_codes.shape[0], k, False)
    return ops.gemm_nvfp4(a, w, bias, epilogue=epilogue)


def _attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    return ops.attention(q, k, v, scale=scale)


def _attention_bnsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    scale: Optional[float] = None) -> torch.Tensor:
    return h3_attention_bnsd(q, k, v, scale=scale)


def _rmsnorm_modulate(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float,
                      row_sel: Optional[torch.Tensor] = None) -> torch.Tensor:
    return ops.rmsnorm_modulate(x.contiguous(), weight, shift, scale, eps, row_sel=row_sel)


def _rmsnorm_modulate_quant_i8(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                               eps: float, row_sel: Optional[torch.Tensor] = None,
                               convrot_group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.rmsnorm_modulate_quant_i8(x, weight, shift, scale, eps, row_sel=row_sel, convrot_group=convrot_group)


# ----------------------------------------------------------------------------- registration

quant_i8_rows = torch.library.custom_op("h3b::quant_i8_rows", mutates_args=(), device_types="cuda")(_quant_i8_rows)
gemm_i8 = torch.library.custom_op("h3b::gemm_i8", mutates_args=(), device_types="cuda")(_gemm_i8)
quant_nvfp4 = torch.library.custom_op("h3b::quant_nvfp4", mutates_args=(), device_types="cuda")(_quant_nvfp4)
gemm_nvfp4 = torch.library.custom_op("h3b::gemm_nvfp4", mutates_args=(), device_types="cuda")(_gemm_nvfp4)
gelu_amax_scan = torch.library.custom_op("h3b::gelu_amax_scan", mutates_args=("ymax2",),
                                         device_types="cuda")(_gelu_amax_scan)
quant_nvfp4_gelu = torch.library.custom_op("h3b::quant_nvfp4_gelu", mutates_args=(),
                                           device_types="cuda")(_quant_nvfp4_gelu)
attention = torch.library.custom_op("h3b::attention", mutates_args=(), device_types="cuda")(_attention)
attention_bnsd = torch.library.custom_op("h3b::attention_bnsd", mutates_args=(),
                                         device_types="cuda")(_attention_bnsd)
rmsnorm_modulate = torch.library.custom_op("h3b::rmsnorm_modulate", mutates_args=(),
                                           device_types="cuda")(_rmsnorm_modulate)
rmsnorm_modulate_quant_i8 = torch.library.custom_op("h3b::rmsnorm_modulate_quant_i8", mutates_args=(),
                                                    device_types="cuda")(_rmsnorm_modulate_quant_i8)


@quant_i8_rows.register_fake
def _(x, convrot_group=0):
    m, k = _rows_of(x), x.shape[-1]
    return x.new_empty((m, k), dtype=torch.int8), x.new_empty((m,), dtype=torch.float32)


@gemm_i8.register_fake
def _(q, xs, w, ws, bias=None, epilogue=0):
    return q.new_empty((q.shape[0], _gemm_cols(w.shape[0], epilogue)), dtype=torch.bfloat16)


@quant_nvfp4.register_fake
def _(x, hi_first=False):
    m, k = _rows_of(x), x.shape[-1]
    sf_bytes = ops.sf_blocked_bytes(m, k) if m else 0
    return (x.new_empty((m, k // 2), dtype=torch.uint8), x.new_empty((sf_bytes,), dtype=torch.uint8),
            x.new_empty((1,), dtype=torch.float32))


@gelu_amax_scan.register_fake
def _(y, ymax2):
    return None


@quant_nvfp4_gelu.register_fake
def _(y, ymax2, hi_first=False):
    m, k = _rows_of(y), y.shape[-1]
    return (y.new_empty((m, k // 2), dtype=torch.uint8), y.new_empty((ops.sf_blocked_bytes(m, k),), dtype=torch.uint8),
            y.new_empty((1,), dtype=torch.float32))


@gemm_nvfp4.register_fake
def _(a_codes, a_sf, a_gs, w_codes, w_sf, w_gs, bias=None, epilogue=0):
    return a_codes.new_empty((a_codes.shape[0], _gemm_cols(w_codes.shape[0], epilogue)), dtype=torch.bfloat16)


@attention.register_fake
def _(q, k, v, scale=None):
    return q.new_empty(tuple(q.shape), dtype=torch.bfloat16)


@attention_bnsd.register_fake
def _(q, k, v, scale=None):
    return q.new_empty(tuple(q.shape), dtype=torch.bfloat16)


@rmsnorm_modulate.register_fake
def _(x, weight, shift, scale, eps, row_sel=None):
    return x.new_empty((_rows_of(x), x.shape[-1]), dtype=torch.bfloat16)


@rmsnorm_modulate_quant_i8.register_fake
def _(x, weight, shift, scale, eps, row_sel=None, convrot_group=0):
    m, hidden = _rows_of(x), x.shape[-1]
    return x.new_empty((m, hidden), dtype=torch.int8), x.new_empty((m,), dtype=torch.float32)
