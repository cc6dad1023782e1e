"""A DiT block exported to a Comfy-quant safetensors file and loaded back
(load/safetensors_quant.py:25-146) runs bit-identically to the original."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt,act", [("nvfp4", "swiglu"), ("int8_tensorwise", "gelu")])
def test_block_round_trip_bit_exact(cuda, tmp_path, fmt, act):
    from minixmax_h3_b200 import checkpoint as ck
    from minixmax_h3_b200.block import DiTBlock, RopeSpec, init_block_random

    def make():
        return DiTBlock(512, 4, 128, 1024, 256, 1e-6, 1e-6, dtype=torch.bfloat16, device=cuda, mlp_act=act)

    blk = make()
    init_block_random(blk, fmt, torch.Generator(device=cuda).manual_seed(0))
    dense, quant = ck.export_checkpoint(blk)
    path = tmp_path / "block.safetensors"
    ck.save_checkpoint(path, dense, quant)
    blk2 = make()
    missing, unexpected = ck.load_checkpoint(blk2, path, device=cuda)
    assert missing == [] and unexpected == []

    pos = RopeSpec.grid_positions(2, 16, 16)
    rope = RopeSpec.build(pos, device=cuda)
    s = pos.shape[0]
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(s, 512, generator=g, device=cuda).to(torch.bfloat16)
    t_emb = torch.randn(1, 256, generator=g, device=cuda).to(torch.bfloat16)
    segs = [(0, 64, 1), (64, s, 0)]
    y1 = blk(x.clone(), t_emb, segs, rope)
    y2 = blk2(x.clone(), t_emb, segs, rope)
    assert torch.equal(y1, y2)
