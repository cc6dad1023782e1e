"""CPU: the ``torch.ops.h3b.*`` custom operators (minixmax_h3_b200/torch_ops.py)
— registration, refusal of non-CUDA tensors, the fake implementations' shapes
(what torch's tracing sees), a traced graph, and the forwarding to ``ops``
with the kernels replaced by recording stand-ins.  The kernels behind them
are covered by the GPU parity tests of ``ops``."""
from __future__ import annotations

from typing import Optional

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from minixmax_h3_b200 import ops
from minixmax_h3_b200 import torch_ops as T

BF16, I8, U8, F32 = torch.bfloat16, torch.int8, torch.uint8, torch.float32
OPS = ("quant_i8_rows", "gemm_i8", "quant_nvfp4", "gemm_nvfp4", "attention", "attention_bnsd",
       "rmsnorm_modulate", "rmsnorm_modulate_quant_i8", "gelu_amax_scan", "quant_nvfp4_gelu")


def test_registered_and_refused_on_cpu():
    for name in OPS:
        assert hasattr(torch.ops.h3b, name), name
    with pytest.raises(NotImplementedError):
        torch.ops.h3b.quant_i8_rows(torch.zeros(2, 64, dtype=BF16), 0)
    with pytest.raises(NotImplementedError):
        torch.ops.h3b.attention(*(torch.zeros(4, 1, 128, dtype=BF16) for _ in range(3)), None)


def test_fake_shapes():
    m, k, n, hidden = 300, 512, 384, 256
    with FakeTensorMode():
        def t(*shape, dtype):
            return torch.empty(*shape, dtype=dtype, device="cuda")

        x = t(m, k, dtype=BF16)
        q, s = torch.ops.h3b.quant_i8_rows(x, 256)
        assert (q.shape, q.dtype, s.shape, s.dtype) == ((m, k), I8, (m,), F32)
        args = (q, s, t(n, k, dtype=I8), t(n, dtype=F32), None)
        y = torch.ops.h3b.gemm_i8(*args, ops.EPI_GELU)
        assert (y.shape, y.dtype, y.device.type) == ((m, n), BF16, "cuda")
        assert torch.ops.h3b.gemm_i8(*args, ops.EPI_SWIGLU).shape == (m, n // 2)
        with pytest.raises(ValueError):
            torch.ops.h3b.gemm_i8(*args, ops.EPI_GATE_RES)

        c, sf, gs = torch.ops.h3b.quant_nvfp4(x, False)
        assert (c.shape, c.dtype, sf.shape, sf.dtype, gs.shape) == ((m, k // 2), U8, (ops.sf_blocked_bytes(m, k),),
                                                                   U8, (1,))
        w_sf = t(ops.sf_blocked_bytes(n, k), dtype=U8)
        y = torch.ops.h3b.gemm_nvfp4(c, sf, gs, t(n, k // 2, dtype=U8), w_sf, t(1, dtype=F32), None, 0)
        assert (y.shape, y.dtype) == ((m, n), BF16)

        o = torch.ops.h3b.attention(t(77, 2, 128, dtype=BF16), t(129, 2, 128, dtype=BF16),
                                    t(129, 2, 128, dtype=BF16), 0.1)
        assert (o.shape, o.dtype) == ((77, 2, 128), BF16)
        o = torch.ops.h3b.attention_bnsd(t(1, 2, 77, 128, dtype=BF16), t(1, 2, 129, 128, dtype=BF16),
                                         t(1, 2, 129, 128, dtype=BF16), None)
        assert o.shape == (1, 2, 77, 128)

        xh = t(m, hidden, dtype=BF16)
        tab = (t(hidden, dtype=BF16), t(3, hidden, dtype=BF16), t(3, hidden, dtype=BF16), 1e-6, t(m, dtype=torch.int32))
        h = torch.ops.h3b.rmsnorm_modulate(xh, *tab)
        assert (h.shape, h.dtype) == ((m, hidden), BF16)
        q, s = torch.ops.h3b.rmsnorm_modulate_quant_i8(xh, *tab, 256)
        assert (q.shape, q.dtype, s.shape) == ((m, hidden), I8, (m,))


def test_traced_graph_holds_the_operators():
    """A function of the operators traces (on meta tensors, through the fake
    implementations) to a graph of h3b calls, by make_fx and by torch.compile
    with fullgraph=True, as the reference's custom op is meant to
    (ops/gather_fa.py:195-206)."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def linear_w4a4(x, w_codes, w_sf, w_gs):
        c, sf, gs = torch.ops.h3b.quant_nvfp4(x, False)
        return torch.ops.h3b.gemm_nvfp4(c, sf, gs, w_codes, w_sf, w_gs, None, ops.EPI_GELU)

    args = (torch.empty(300, 512, dtype=BF16, device="meta"), torch.empty(384, 256, dtype=U8, device="meta"),
            torch.empty(ops.sf_blocked_bytes(384, 512), dtype=U8, device="meta"),
            torch.empty(1, dtype=F32, device="meta"))
    g = make_fx(linear_w4a4)(*args)
    called = [str(nd.target) for nd in g.graph.nodes if nd.op == "call_function"]
    assert "h3b.quant_nvfp4.default" in called and "h3b.gemm_nvfp4.default" in called
    assert linear_w4a4(*args).shape == (300, 384)
    # torch.compile captures both operators in one graph (no graph break)
    compiled = torch.compile(linear_w4a4, backend="eager", fullgraph=True)
    assert compiled(*args).shape == (300, 384)


def test_forwarding_to_ops(monkeypatch):
    """The implementations hand their tensors to the ops wrappers unchanged:
    NVFP4 operands rebuilt with rows, K and the tensor cores' nibble order,
    epilogues passed through, the in-place epilogue and mismatched K refused."""
    seen = {}

    def fake_gemm_nvfp4(a, w, bias, *, epilogue):
        seen["nvfp4"] = (a, w, bias, epilogue)
        return torch.zeros(a.rows, w.rows)

    def fake_gemm_i8(q, xs, w, ws, bias, *, epilogue):
        seen["i8"] = (q, xs, w, ws, bias, epilogue)
        return torch.zeros(q.shape[0], w.shape[0])

    def fake_quant_nvfp4(x, *, hi_first):
        return ops.NVFP4Tensor(torch.ones(3, 8, dtype=U8), torch.ones(4, dtype=U8), torch.ones(1), 3, 16, hi_first)

    monkeypatch.setattr(ops, "gemm_nvfp4", fake_gemm_nvfp4)
    monkeypatch.setattr(ops, "gemm_i8", fake_gemm_i8)
    monkeypatch.setattr(ops, "quant_nvfp4", fake_quant_nvfp4)

    a_codes, a_sf, a_gs = torch.zeros(5, 32, dtype=U8), torch.zeros(7, dtype=U8), torch.ones(1)
    w_codes, w_sf, w_gs = torch.zeros(6, 32, dtype=U8), torch.zeros(9, dtype=U8), torch.full((1,), 2.0)
    bias = torch.zeros(6, dtype=BF16)
    T._gemm_nvfp4(a_codes, a_sf, a_gs, w_codes, w_sf, w_gs, bias, ops.EPI_SWIGLU)
    a, w, b, epi = seen["nvfp4"]
    assert (a.rows, a.k, a.hi_first, w.rows, w.k, w.hi_first) == (5, 64, False, 6, 64, False)
    assert a.codes is a_codes and a.sf is a_sf and a.gs is a_gs and w.gs is w_gs and b is bias
    assert epi == ops.EPI_SWIGLU
    with pytest.raises(ValueError):
        T._gemm_nvfp4(a_codes, a_sf, a_gs, torch.zeros(6, 16, dtype=U8), w_sf, w_gs, None, 0)
    with pytest.raises(ValueError):
        T._gemm_nvfp4(a_codes, a_sf, a_gs, w_codes, w_sf, w_gs, None, ops.EPI_GATE_RES)

    q, xs, wi, ws = torch.zeros(5, 64, dtype=I8), torch.ones(5), torch.zeros(6, 64, dtype=I8), torch.ones(6)
    T._gemm_i8(q, xs, wi, ws, None, ops.EPI_GELU)
    assert all(got is want for got, want in zip(seen["i8"][:4], (q, xs, wi, ws))) and seen["i8"][5] == ops.EPI_GELU
    with pytest.raises(ValueError):
        T._gemm_i8(q, xs, wi, ws, None, ops.EPI_GATE_RES)

    codes, sf, gs = T._quant_nvfp4(torch.zeros(3, 16, dtype=BF16), True)
    assert codes.shape == (3, 8) and sf.shape == (4,) and gs.shape == (1,)


def test_dispatch_mechanics_on_cpu(monkeypatch):
    """torch.library's calling convention for these implementations (optional
    tensors given as None, int epilogues, tuple results, fresh outputs),
    exercised through CPU-device twins registered in a test namespace around
    the same implementation functions, with the kernels replaced by
    recorders."""

    def fake_quant_nvfp4(x, *, hi_first):
        m, k = x.shape
        return ops.NVFP4Tensor(torch.zeros(m, k // 2, dtype=U8), torch.zeros(ops.sf_blocked_bytes(m, k), dtype=U8),
                               torch.ones(1), m, k, hi_first)

    def fake_gemm_nvfp4(a, w, bias, *, epilogue):
        return torch.full((a.rows, w.rows // (2 if epilogue == ops.EPI_SWIGLU else 1)), float(a.k),
                          dtype=BF16)

    def fake_quant_i8(x, *, convrot_group=0, x_rot_out=None):
        return torch.full(x.shape, convrot_group % 127, dtype=I8), torch.ones(x.shape[0])

    monkeypatch.setattr(ops, "quant_nvfp4", fake_quant_nvfp4)
    monkeypatch.setattr(ops, "gemm_nvfp4", fake_gemm_nvfp4)
    monkeypatch.setattr(ops, "quant_i8_rows", fake_quant_i8)

    @torch.library.custom_op("h3btest::quant_nvfp4", mutates_args=(), device_types="cpu")
    def tq(x: torch.Tensor, hi_first: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return T._quant_nvfp4(x, hi_first)

    @torch.library.custom_op("h3btest::gemm_nvfp4", mutates_args=(), device_types="cpu")
    def tg(a_codes: torch.Tensor, a_sf: torch.Tensor, a_gs: torch.Tensor, w_codes: torch.Tensor, w_sf: torch.Tensor,
           w_gs: torch.Tensor, bias: Optional[torch.Tensor] = None, epilogue: int = 0) -> torch.Tensor:
        return T._gemm_nvfp4(a_codes, a_sf, a_gs, w_codes, w_sf, w_gs, bias, epilogue)

    @torch.library.custom_op("h3btest::quant_i8_rows", mutates_args=(), device_types="cpu")
    def ti(x: torch.Tensor, convrot_group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        return T._quant_i8_rows(x, convrot_group)

    x = torch.zeros(300, 512, dtype=BF16)
    c, sf, gs = torch.ops.h3btest.quant_nvfp4(x, False)
    assert (c.shape, sf.shape, gs.shape) == ((300, 256), (ops.sf_blocked_bytes(300, 512),), (1,))
    w = (torch.zeros(384, 256, dtype=U8), torch.zeros(ops.sf_blocked_bytes(384, 512), dtype=U8), torch.ones(1))
    y = torch.ops.h3btest.gemm_nvfp4(c, sf, gs, *w, None, ops.EPI_SWIGLU)
    assert y.shape == (300, 192) and y.dtype == BF16 and float(y[0, 0]) == 512.0
    y = torch.ops.h3btest.gemm_nvfp4(c, sf, gs, *w, torch.zeros(384, dtype=BF16), 0)
    assert y.shape == (300, 384)
    q, s = torch.ops.h3btest.quant_i8_rows(x, 256)
    assert q.shape == (300, 512) and int(q[0, 0]) == 256 % 127 and s.shape == (300,)
