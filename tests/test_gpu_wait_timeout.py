"""GPU: the bounded-wait unwind, exercised in the allowed form.

h3b_selftest_wait_timeout launches the NVFP4 GEMM with its producer issuing no
loads: no copy is ever in flight, and the MMA thread's wait for the first K
slab is a wait on a barrier that nothing will complete.  The wait must run
out after its budget (2 s), and the device status must name the timeout and
the site of the first wait to run out (3: the MMA thread's wait for the slab;
4: an epilogue warp's wait for the accumulator; 7: a scale writer's wait for
the slab's scales — all start together on barriers nothing completes).  The
kernel must return without writing its output, and the next ordinary launch
on the same context must give the same bits as before.  No trap, no fault, no unbounded wait.  (The
reference's counterparts are host-side timeouts: runtime/dist.py:43,99-116.)"""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

H3B_ERR_DEVICE_TIMEOUT = 6
CONSUMER_SITES = {3, 4, 7}  # MMA slab wait, epilogue accumulator wait, scale-writer wait


def test_bounded_wait_runs_out_and_the_context_stays_usable(cuda):
    from minixmax_h3_b200 import _lib, ops

    g = torch.Generator(device=cuda).manual_seed(0)
    m, n, k = 128, 192, 512
    a = ops.quant_nvfp4(torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16))
    w = ops.quant_nvfp4((0.02 * torch.randn(n, k, generator=g, device=cuda)).to(torch.bfloat16))
    before = ops.gemm_nvfp4(a, w)
    assert _lib.device_status(clear=True) == (0, 0, 0, 0)

    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    t0 = time.monotonic()
    _lib.call("h3b_selftest_wait_timeout", a.codes.data_ptr(), a.sf.data_ptr(), a.gs.data_ptr(), w.codes.data_ptr(),
              w.sf.data_ptr(), w.gs.data_ptr(), y.data_ptr(), m, n, k,
              torch.cuda.current_stream(cuda).cuda_stream)
    code, site, _info, block = _lib.device_status(clear=True)  # synchronises
    elapsed = time.monotonic() - t0
    assert code == H3B_ERR_DEVICE_TIMEOUT and site in CONSUMER_SITES and block == 0, (code, site, block)
    assert 1.5 <= elapsed <= 20.0, elapsed  # the 2 s budget, not a hang
    assert torch.isnan(y.float()).all()  # the unwound kernel wrote nothing

    after = ops.gemm_nvfp4(a, w)
    assert torch.equal(after, before)
    assert _lib.device_status(clear=True) == (0, 0, 0, 0)
