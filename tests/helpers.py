"""Test helpers: golden fixture loading and the float acceptance bar."""
from __future__ import annotations

from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / name, weights_only=False)


def assert_close_bf16(got: torch.Tensor, want: torch.Tensor, max_abs: float = 2e-2, min_cos: float = 0.9995):
    """The hot path's float acceptance bar for bf16 outputs.

    Error is |got - want| / max(1, |want|): an absolute 2e-2 bound for
    |want| <= 1 that becomes relative above 1, because one bf16 ulp exceeds
    2e-2 once |want| >= 4 (e.g. 0.0625 at 16) and a pure absolute bound would
    then test the output rounding instead of the kernel.  Cosine similarity
    over the whole tensor must be >= 0.9995.
    """
    g = got.detach().float().cpu().reshape(-1)
    w = want.detach().float().cpu().reshape(-1)
    assert torch.isfinite(g).all(), "non-finite output"
    diff = (g - w).abs()
    err = (diff / w.abs().clamp(min=1.0)).max().item()
    raw = diff.max().item()
    cos = torch.nn.functional.cosine_similarity(g.double(), w.double(), dim=0).item()
    assert err <= max_abs and cos >= min_cos, (
        f"scaled max_abs={err:.4g} (<= {max_abs}) cos={cos:.6f} (>= {min_cos}); raw max_abs={raw:.4g}, "
        f"{int((diff > 2e-2).sum())} of {diff.numel()} elements above an absolute 2e-2")
    return err, cos, raw
