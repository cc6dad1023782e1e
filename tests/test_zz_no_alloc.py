"""The allocation-free entry point h3b_rmsnorm_modulate_quant_nvfp4_noalloc,
called through the C ABI, against the two-call path it replaces
(h3b_rmsnorm_modulate then h3b_quant_nvfp4, with caller buffers for the
modulated rows and their |max|).  It is for callers that may not allocate
device memory while they run; its scratch is a fixed array inside the
library, shared by every call on the device.  Two calls in a row with
different inputs and sizes check that nothing of the first call's scratch
leaks into the second.  The bar is the quantisers' own: bit-exact codes,
block scales and global scale."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed: int, m: int, hidden: int, device, *, gain: float = 1.0, pad: int = 0, row_sel: bool = True):
    """x [m, hidden] (a column slice of a [m, hidden + pad] tensor when pad > 0,
    so its row stride exceeds hidden), the norm weight and adaLN tables scaled
    by `gain`, and per-token table rows (or None)."""
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, hidden + pad, generator=g) * 2).to(torch.bfloat16).to(device)[:, :hidden]
    w = (gain * (1 + 0.1 * torch.randn(hidden, generator=g))).to(torch.bfloat16).to(device)
    tab = (gain * 0.2 * torch.randn(2, 2 * hidden, generator=g)).to(torch.bfloat16).to(device)
    sel = torch.randint(-1, 2, (m,), generator=g, dtype=torch.int32).to(device) if row_sel else None
    return x, w, tab[:, :hidden], tab[:, hidden:], sel


def _noalloc(x, w, shift, scale, sel, hi_first):
    from minixmax_h3_b200 import ops
    from minixmax_h3_b200._lib import call

    m, hidden = x.shape
    codes = torch.empty(m, hidden // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(ops.sf_blocked_bytes(m, hidden), dtype=torch.uint8, device=x.device)
    gs = torch.empty(1, dtype=torch.float32, device=x.device)
    call("h3b_rmsnorm_modulate_quant_nvfp4_noalloc", x.data_ptr(), m, hidden, x.stride(0), w.data_ptr(),
         shift.data_ptr(), scale.data_ptr(), shift.stride(0), None if sel is None else sel.data_ptr(), 1e-6,
         codes.data_ptr(), sf.data_ptr(), gs.data_ptr(), 1 if hi_first else 0,
         torch.cuda.current_stream(x.device).cuda_stream)
    return codes, sf, gs


def _two_calls(x, w, shift, scale, sel, hi_first):
    from minixmax_h3_b200 import ops

    amax = torch.zeros(1, dtype=torch.float32, device=x.device)
    m, hidden = x.shape
    h = torch.empty(m, x.stride(0), dtype=torch.bfloat16, device=x.device)[:, :hidden]  # x's row stride
    h = ops.rmsnorm_modulate(x, w, shift, scale, 1e-6, row_sel=sel, amax_out=amax, out=h)
    t = ops.quant_nvfp4(h, hi_first=hi_first, amax_t=amax)
    return t.codes, t.sf, t.gs


def test_noalloc_matches_two_call_path(cuda):
    """Two calls in a row.  The second call's |h| max is about ten times
    smaller than the first's (norm weight and tables scaled by 0.1; scaling x
    would not change h, which RMSNorm normalises), so a max left over from the
    first call would give it a wrong global scale and wrong codes."""
    gs_seen = []
    for seed, (m, hidden), hi_first, gain in ((0, (300, 3072), True, 1.0), (1, (129, 1024), False, 0.1)):
        args = _inputs(seed, m, hidden, cuda, gain=gain)
        got = _noalloc(*args, hi_first)
        want = _two_calls(*args, hi_first)
        for a, b in zip(got, want):
            assert torch.equal(a, b)
        gs_seen.append(got[2].item())
    assert gs_seen[1] < 0.5 * gs_seen[0], gs_seen


def test_noalloc_wide_row_stride_and_no_row_sel(cuda):
    """x as a column slice of a wider tensor (row stride hidden + 64, which
    the array holds h with) and row_sel NULL (every token on table row 0),
    bit-exact against the two-call path."""
    for seed, row_sel in ((3, True), (4, False)):
        args = _inputs(seed, 200, 1024, cuda, pad=64, row_sel=row_sel)
        assert args[0].stride(0) == 1024 + 64
        for a, b in zip(_noalloc(*args, True), _two_calls(*args, True)):
            assert torch.equal(a, b)


def test_noalloc_rejects_sizes_beyond_its_array(cuda):
    """Rows beyond the 16 MiB array: H3B_ERR_SHAPE before anything is
    queued (the output pointers are valid but far too small; the entry point
    never reaches them).  A null output is refused as such, also before any
    work."""
    from minixmax_h3_b200._lib import H3bError, call

    x, w, shift, scale, sel = _inputs(2, 64, 1024, cuda)
    codes = torch.empty(64, 512, dtype=torch.uint8, device=cuda)
    sf = torch.empty(128 * 64, dtype=torch.uint8, device=cuda)
    gs = torch.empty(1, dtype=torch.float32, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    too_many = (16 << 20) // (2 * 1024) + 1  # rows of 1024 bf16 beyond the 16 MiB array
    with pytest.raises(H3bError) as e:
        call("h3b_rmsnorm_modulate_quant_nvfp4_noalloc", x.data_ptr(), too_many, 1024, 1024, w.data_ptr(),
             shift.data_ptr(), scale.data_ptr(), shift.stride(0), sel.data_ptr(), 1e-6, codes.data_ptr(),
             sf.data_ptr(), gs.data_ptr(), 1, stream)
    assert e.value.code == 1  # H3B_ERR_SHAPE
    with pytest.raises(H3bError) as e:
        call("h3b_rmsnorm_modulate_quant_nvfp4_noalloc", x.data_ptr(), 64, 1024, 1024, w.data_ptr(),
             shift.data_ptr(), scale.data_ptr(), shift.stride(0), sel.data_ptr(), 1e-6, None, sf.data_ptr(),
             gs.data_ptr(), 1, stream)
    assert e.value.code == 8  # H3B_ERR_ARG
