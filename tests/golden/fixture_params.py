"""Seeded weights of the DiT-block golden fixtures (dit_block_*.pt).

The fixtures store only the seed of their weights; this module rebuilds them.
It imports nothing but torch, so the GPU box's checks (the tests and the
benchmark's parity check) can rebuild a fixture's block without the oracle.
"""
from __future__ import annotations

import torch


def block_params(g: torch.Generator, hidden: int, heads: int, ffn_out: int, ffn_in: int, t_dim: int) -> dict:
    """Seeded block weights (bf16).  The fixtures store only the seed; tests
    call this again with the same generator state to rebuild them."""
    inner = heads * 128
    p = {
        "qkv_w": torch.randn(3 * inner, hidden, generator=g) * 0.02,
        "out_w": torch.randn(hidden, inner, generator=g) * 0.02,
        "fc1_w": torch.randn(ffn_out, hidden, generator=g) * 0.02,
        "fc2_w": torch.randn(hidden, ffn_in, generator=g) * 0.02,
        "adaln_w": torch.randn(6 * hidden * 3, t_dim, generator=g) * 0.02,
        "adaln_b": torch.randn(6 * hidden * 3, generator=g) * 0.02,
        "norm1_w": 1.0 + 0.1 * torch.randn(hidden, generator=g),
        "norm2_w": 1.0 + 0.1 * torch.randn(hidden, generator=g),
        "q_norm_w": 1.0 + 0.1 * torch.randn(128, generator=g),
        "k_norm_w": 1.0 + 0.1 * torch.randn(128, generator=g),
    }
    return {k: v.to(torch.bfloat16) for k, v in p.items()}


def block_fixture_params(fix: dict) -> dict:
    """Rebuilds the weights of a block fixture from its seed."""
    g = torch.Generator().manual_seed(fix["seed"])
    hidden, ffn = fix["hidden"], 4 * fix["hidden"]
    ffn_out = ffn if fix["mlp_act"] == "gelu" else 2 * ffn
    return block_params(g, hidden, fix["heads"], ffn_out, ffn, fix["t_dim"])
