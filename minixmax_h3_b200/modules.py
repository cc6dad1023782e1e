"""Drop-in ``nn.Linear`` replacement and the ``operations`` namespace.

Mirrors the reference's modules/linear.py (QuantLinear 65-210, Linear 35-62,
RMSNorm 15-32, NpuOps 248-252): same constructor, ``from_quant_tensors``,
``set_quant``, ``prepare_cube`` and ``forward`` contract, same Comfy quant
formats ("int8_tensorwise" W8A8 with per-output-channel fp32 weight scales,
"nvfp4" with packed e2m1 codes, blocked e4m3 block scales and an fp32
per-tensor scale).  Compute goes to libh3b.so; there is no CPU path.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .ops import EPI_STORE, NVFP4Tensor
from .timing import TIMER


class RMSNorm(nn.Module):
    """RMSNorm over the last dim (modules/linear.py:15-32)."""

    def __init__(self, dim: int, eps: float = 1e-5, dtype=None, device=None, **_):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype or torch.bfloat16, device=device),
                                   requires_grad=False)
        self._no_mod = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            raise TypeError("RMSNorm kernel expects bf16 activations")
        hidden = x.shape[-1]
        if self._no_mod is None or self._no_mod.device != x.device:
            self._no_mod = torch.zeros(hidden, dtype=torch.bfloat16, device=x.device)
        sel = torch.full((x.numel() // hidden,), -1, dtype=torch.int32, device=x.device)
        out = ops.rmsnorm_modulate(x, self.weight.to(x.device), self._no_mod, self._no_mod, self.eps, row_sel=sel)
        return out.view_as(x)


class Linear(nn.Module):
    """Dense bf16 Linear with Comfy ``operations.Linear`` constructor kwargs
    (modules/linear.py:35-62).  Used only for the 1-row adaLN projection; the
    quantised projections are QuantLinear."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, dtype=None, device=None, **_):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        dt = dtype or torch.bfloat16
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=dt, device=device),
                                   requires_grad=False)
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=dt, device=device), requires_grad=False)
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight.to(dtype=x.dtype, device=x.device)
        b = self.bias.to(dtype=x.dtype, device=x.device) if self.bias is not None else None
        return F.linear(x, w, b)


@dataclass
class QuantizedRows:
    """An activation already quantised for an INT8 QuantLinear: codes
    q [m, K] int8 and per-row scales [m] fp32, rotated by ConvRot before
    quantisation when convrot_group is 256 — e.g. from
    ops.rmsnorm_modulate_quant_i8.  Accepted by the INT8 forward paths in
    place of the bf16 input."""
    q: torch.Tensor
    scale: torch.Tensor
    convrot_group: int = 0

    @property
    def shape(self) -> torch.Size:
        return self.q.shape

    @property
    def device(self) -> torch.device:
        return self.q.device


class QuantLinear(nn.Module):
    """INT8 W8A8 / NVFP4 W4A4 Linear on tcgen05 (modules/linear.py:65-210)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, dtype=None, device=None, **_):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.quant_format: Optional[str] = None
        self.convrot = False
        self.group_size = 256
        self._compute_dtype = dtype or torch.bfloat16
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=self._compute_dtype, device=device),
                                   requires_grad=False)
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=self._compute_dtype, device=device),
                                     requires_grad=False)
        else:
            self.register_parameter("bias", None)
        self.register_buffer("weight_i8", None, persistent=False)
        self.register_buffer("weight_u8", None, persistent=False)
        self.register_buffer("weight_scale", None, persistent=False)
        self.register_buffer("weight_scale_2", None, persistent=False)
        self.register_buffer("pre_quant_scale", None, persistent=False)
        self.weight_layout = "nk"
        self._w_nvfp4: Optional[NVFP4Tensor] = None
        self._row_perm: Optional[torch.Tensor] = None  # set by interleave_swiglu

    @classmethod
    def from_quant_tensors(cls, weight: torch.Tensor, *, meta: dict[str, Any],
                           weight_scale: Optional[torch.Tensor] = None,
                           weight_scale_2: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                           pre_quant_scale: Optional[torch.Tensor] = None, device=None,
                           compute_dtype=torch.bfloat16) -> "QuantLinear":
        fmt = meta.get("format")
        if fmt == "nvfp4":
            out_f, packed_k = weight.shape
            in_f = packed_k * 2
        else:
            out_f, in_f = weight.shape
        m = cls(in_f, out_f, bias=bias is not None, dtype=compute_dtype, device=device)
        m.set_quant(weight, meta=meta, weight_scale=weight_scale, weight_scale_2=weight_scale_2, bias=bias,
                    pre_quant_scale=pre_quant_scale, device=device)
        return m

    def set_quant(self, weight: torch.Tensor, *, meta: dict[str, Any], weight_scale: Optional[torch.Tensor] = None,
                  weight_scale_2: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                  pre_quant_scale: Optional[torch.Tensor] = None, device=None) -> None:
        """Adopts checkpoint tensors (modules/linear.py:138-169)."""
        self.quant_format = meta.get("format")
        self.convrot = bool(meta.get("convrot", False))
        self.group_size = int(meta.get("convrot_groupsize", 256))
        # ConvRot only changes the INT8 path (ops/int8_convrot.py:139-140);
        # the NVFP4 path ignores the flag, as the reference's does.
        if self.convrot and self.quant_format == "int8_tensorwise" and self.group_size != 256:
            raise NotImplementedError(f"ConvRot group size {self.group_size}: this build rotates 256-column groups")
        self.weight = nn.Parameter(torch.empty(0, device=device), requires_grad=False)
        if self.quant_format == "int8_tensorwise":
            self.weight_i8 = weight.to(device=device, dtype=torch.int8).contiguous()
            self.weight_scale = weight_scale.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
            self.out_features, self.in_features = self.weight_i8.shape
        elif self.quant_format == "nvfp4":
            self.weight_u8 = weight.to(device=device).view(torch.uint8).contiguous()
            self.weight_scale = weight_scale.to(device=device).view(torch.uint8).reshape(-1).contiguous()
            ws2 = weight_scale_2.to(device=device)
            if ws2.dtype != torch.float32:
                ws2 = ws2.float()
            self.weight_scale_2 = ws2.reshape(1).contiguous()
            self.out_features = self.weight_u8.shape[0]
            self.in_features = self.weight_u8.shape[1] * 2
            expect = ops.sf_blocked_bytes(self.out_features, self.in_features)
            if self.weight_scale.numel() != expect:
                raise ValueError(f"nvfp4 block scales: expected {expect} blocked bytes, got {self.weight_scale.numel()}")
        else:
            raise ValueError(f"unsupported quant format: {self.quant_format}")
        self.weight_layout = "nk"
        self._w_nvfp4 = None
        self._row_perm = None
        if bias is not None:
            self.bias = nn.Parameter(bias.to(device=device, dtype=self._compute_dtype), requires_grad=False)
        if pre_quant_scale is not None:
            self.pre_quant_scale = pre_quant_scale.to(device=device)

    def prepare_cube(self) -> None:
        """One-time device repack after the weights reach the GPU
        (modules/linear.py:171-181).  INT8 needs none: the GEMM reads the [N, K]
        weight K-major as stored.  NVFP4 codes are swapped from the checkpoint's
        hi-first nibble order to the tensor cores' lo-first order; the blocked
        scales are consumed as stored."""
        if self.quant_format == "nvfp4" and self._w_nvfp4 is None:
            if not self.weight_u8.is_cuda:
                raise RuntimeError("prepare_cube needs the weights on the GPU")
            codes = ops.swap_nibbles(self.weight_u8)
            self._w_nvfp4 = NVFP4Tensor(codes, self.weight_scale, self.weight_scale_2, self.out_features,
                                        self.in_features, hi_first=False)
            self.weight_layout = "nk_lo_first"

    def interleave_swiglu(self) -> None:
        """One-time reorder of an fc1 weight (rows = [gate; up]) into the
        32-row interleave the fused SwiGLU epilogue reads (ops.swiglu_
        interleave_perm): codes, per-row scales, block scales and bias move
        together.  forward() restores the reference's column order; use
        forward_fused(epilogue=EPI_SWIGLU) for the fused activation."""
        if self._row_perm is not None:
            return
        perm = ops.swiglu_interleave_perm(self.out_features, device=self.weight_scale.device)
        if self.quant_format == "int8_tensorwise":
            self.weight_i8 = self.weight_i8[perm].contiguous()
            self.weight_scale = self.weight_scale[perm].contiguous()
        elif self.quant_format == "nvfp4":
            self.weight_u8 = self.weight_u8[perm].contiguous()
            self.weight_scale = ops.permute_blocked_rows(self.weight_scale, self.out_features, self.in_features,
                                                         perm)
            self._w_nvfp4 = None
        else:
            raise RuntimeError("interleave_swiglu needs quantised weights")
        if self.bias is not None and self.bias.numel():
            self.bias = nn.Parameter(self.bias.data[perm].contiguous(), requires_grad=False)
        self._row_perm = perm
        self._inv_perm = torch.argsort(perm)

    def _quant_i8_input(self, x) -> tuple[torch.Tensor, torch.Tensor]:
        group = self.group_size if self.convrot else 0
        if isinstance(x, QuantizedRows):
            if x.convrot_group != group:
                raise ValueError(f"input quantised with ConvRot group {x.convrot_group}, layer expects {group}")
            return x.q, x.scale
        return ops.quant_i8_rows(x, convrot_group=group)

    def _bias(self, x) -> Optional[torch.Tensor]:
        return None if self.bias is None or self.bias.numel() == 0 else self.bias.to(torch.bfloat16)

    def _pre_scale(self, x, amax: Optional[torch.Tensor]):
        """The reference multiplies a layer's input by ``pre_quant_scale``
        before quantising it (modules/linear.py:184-185).  Returns the scaled
        input and the amax still valid for it: a max of the unscaled input
        (from the producing kernel) no longer is, so it is dropped."""
        if self.pre_quant_scale is None:
            return x, amax
        if isinstance(x, QuantizedRows):
            raise ValueError("this layer has a pre_quant_scale: it needs the bf16 input, not rows already quantised")
        return x * self.pre_quant_scale.to(device=x.device, dtype=x.dtype), None

    def forward_fused(self, x: torch.Tensor, *, amax: Optional[torch.Tensor] = None, epilogue: int = EPI_STORE,
                      resid: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
                      row_sel: Optional[torch.Tensor] = None, amax_out: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Quantise x [m, K] bf16 (after ``pre_quant_scale``, when the layer has
        one) and run the GEMM with a fused epilogue.

        amax: precomputed max|x| (fp32 device scalar) for the NVFP4 global
        scale, e.g. from the producing kernel; computed here when None."""
        x, amax = self._pre_scale(x, amax)
        return self._run(x, amax=amax, epilogue=epilogue, resid=resid, gate=gate, row_sel=row_sel,
                         amax_out=amax_out, out=out)

    def forward_gelu_input(self, y: torch.Tensor, ymax2: torch.Tensor, *, epilogue: int = EPI_STORE,
                           resid: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
                           row_sel: Optional[torch.Tensor] = None, amax_out: Optional[torch.Tensor] = None,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """fc2 of the GELU MLP fed fc1's bf16 pre-activation y: the GELU is
        applied inside this layer's NVFP4 input quantiser
        (ops.quant_nvfp4_gelu), so activation and quantisation are one pass
        over y and u = bf16(gelu(y)) is never written.  ymax2: fp32 [2] from
        fc1's EPI_STORE_POSMAX max and ops.gelu_amax_scan (max-reduced across
        ranks).  NVFP4 layers without a pre_quant_scale only."""
        if self.quant_format != "nvfp4" or self.pre_quant_scale is not None:
            raise ValueError("forward_gelu_input needs an NVFP4 layer without a pre_quant_scale")
        self.prepare_cube()
        with TIMER.span("quant"):
            a = ops.quant_nvfp4_gelu(y, ymax2)
        with TIMER.span("gemm", *self._gemm_cost(a.rows)):
            return ops.gemm_nvfp4(a, self._w_nvfp4, self._bias(y), epilogue=epilogue, resid=resid, gate=gate,
                                  row_sel=row_sel, amax_out=amax_out, out=out)

    def _run(self, x, *, amax: Optional[torch.Tensor] = None, epilogue: int = EPI_STORE,
             resid: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
             row_sel: Optional[torch.Tensor] = None, amax_out: Optional[torch.Tensor] = None,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.quant_format == "int8_tensorwise":
            with TIMER.span("quant"):
                q, xs = self._quant_i8_input(x)
            with TIMER.span("gemm", *self._gemm_cost(q.shape[0])):
                return ops.gemm_i8(q, xs, self.weight_i8, self.weight_scale, self._bias(x), epilogue=epilogue,
                                   resid=resid, gate=gate, row_sel=row_sel, amax_out=amax_out, out=out)
        if self.quant_format == "nvfp4":
            self.prepare_cube()
            if isinstance(x, QuantizedRows):
                raise TypeError("an NVFP4 layer needs the bf16 input, not INT8 QuantizedRows")
            with TIMER.span("quant"):
                a = ops.quant_nvfp4(x, amax_t=amax)
            with TIMER.span("gemm", *self._gemm_cost(a.rows)):
                return ops.gemm_nvfp4(a, self._w_nvfp4, self._bias(x), epilogue=epilogue, resid=resid, gate=gate,
                                      row_sel=row_sel, amax_out=amax_out, out=out)
        raise RuntimeError("QuantLinear has no quantised weights (call set_quant first)")

    def _gemm_cost(self, m: int) -> tuple[float, tuple]:
        """(flops, (format, m, n, k)) of one GEMM launch over m rows."""
        return 2.0 * m * self.out_features * self.in_features, (self.quant_format, m, self.out_features,
                                                                 self.in_features)

    def forward_seq2head(self, x: torch.Tensor, recv_ptrs, rank: int, heads: int, *,
                         amax: Optional[torch.Tensor] = None) -> None:
        """QKV projection of this rank's tokens stored straight into every head
        owner's receive buffer (ops.gemm_*_seq2head): the projection and the
        seq->head Ulysses exchange in one kernel."""
        x, amax = self._pre_scale(x, amax)
        if self.quant_format == "int8_tensorwise":
            with TIMER.span("quant"):
                q, xs = self._quant_i8_input(x)
            with TIMER.span("gemm_seq2head", *self._gemm_cost(q.shape[0])):
                ops.gemm_i8_seq2head(q, xs, self.weight_i8, self.weight_scale, self._bias(x), recv_ptrs, rank,
                                     heads)
            return
        if self.quant_format == "nvfp4":
            self.prepare_cube()
            if isinstance(x, QuantizedRows):
                raise TypeError("an NVFP4 layer needs the bf16 input, not INT8 QuantizedRows")
            with TIMER.span("quant"):
                a = ops.quant_nvfp4(x, amax_t=amax)
            with TIMER.span("gemm_seq2head", *self._gemm_cost(a.rows)):
                ops.gemm_nvfp4_seq2head(a, self._w_nvfp4, self._bias(x), recv_ptrs, rank, heads)
            return
        raise RuntimeError("QuantLinear has no quantised weights (call set_quant first)")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """y = x @ W^T (+ bias) through the quantised GEMM; out dtype as the
        reference (x.dtype for bf16/fp16 input, else bf16)."""
        if not x.is_cuda:
            raise RuntimeError("QuantLinear runs on CUDA tensors only (no CPU fallback)")
        if self.pre_quant_scale is not None:
            x = x * self.pre_quant_scale.to(device=x.device, dtype=x.dtype)
        out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else self._compute_dtype
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if self.quant_format == "nvfp4" or x2.dtype != torch.float16:
            x2 = x2.to(torch.bfloat16)
        y = self._run(x2)  # pre_quant_scale applied above, before the dtype cast, as the reference does
        if self._row_perm is not None:  # interleaved for the fused SwiGLU: reference column order
            y = y[:, self._inv_perm]
        return y.to(out_dtype).reshape(*lead, self.out_features)


def decode_comfy_quant(blob: torch.Tensor) -> dict[str, Any]:
    """Comfy ``*.comfy_quant`` JSON blob (the bytes of a uint8 tensor) -> dict
    (modules/linear.py:243-245)."""
    return json.loads(bytes(blob.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()).decode("utf-8"))


class Ops:
    """The ``operations=`` namespace (modules/linear.py:248-252)."""

    Linear = Linear
    RMSNorm = RMSNorm
    QuantLinear = QuantLinear
