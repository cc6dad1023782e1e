"""CPU: host-side layout logic of the package (no kernels launched)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import h3_oracle as O


def test_swiglu_interleave_perm_pairs_gate_and_up():
    from minixmax_h3_b200 import ops

    n = 2 * 192
    perm = ops.swiglu_interleave_perm(n)
    assert sorted(perm.tolist()) == list(range(n))
    ffn = n // 2
    for b in range(ffn // 32):
        for j in range(32):
            assert perm[64 * b + j] == 32 * b + j              # gate column 32b+j
            assert perm[64 * b + 32 + j] == ffn + 32 * b + j   # its up column


def test_permute_blocked_rows_matches_dense_permutation():
    from minixmax_h3_b200 import ops

    g = torch.Generator().manual_seed(0)
    rows, k = 320, 512  # 3 row blocks (last one padded), 32 scale columns
    w = (torch.randn(rows, k, generator=g) * 0.02).to(torch.bfloat16)
    qz = O.nvfp4_quantize(w, hi_first=True)
    perm = ops.swiglu_interleave_perm(rows)
    out = ops.permute_blocked_rows(qz["sf"], rows, k, perm)
    dense = O.from_blocked(qz["sf"].numpy(), rows, k // 16)
    want = O.to_blocked(dense[perm.numpy()])
    assert np.array_equal(out.numpy().reshape(-1), np.asarray(want).reshape(-1))
