"""Comfy-quant checkpoint loading (load/safetensors_quant.py:25-146,
modules/linear.py:105-169, 243-245) on CPU: the metadata encoding, a
synthetic DiT checkpoint in the reference's layout (INT8 with and without
ConvRot, NVFP4 with hi-first codes and blocked scales) written with
safetensors and loaded back into DiTStep / DiTBlock."""
from __future__ import annotations

import pytest
import torch

from oracle import h3_oracle as O


def _nvfp4(w: torch.Tensor) -> dict:
    q = O.nvfp4_quantize(w.to(torch.bfloat16), hi_first=True)
    return {"weight": q["codes"], "weight_scale": q["sf"], "weight_scale_2": q["gs"].reshape(1),
            "meta": {"format": "nvfp4"}}


def _int8(w: torch.Tensor, convrot: bool) -> dict:
    from minixmax_h3_b200.block import quantize_linear_weight

    d = quantize_linear_weight(w, "int8_tensorwise")
    if convrot:
        d["meta"] = {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256}
    return d


def _step(depth: int = 2):
    from minixmax_h3_b200.block import DiTStep

    return DiTStep(hidden=256, heads=2, ffn=512, depth=depth, text_dim=128, device="cpu")


def _synthetic(depth: int = 2, seed: int = 0):
    """dense state-dict entries + quant dicts for a DiTStep(hidden 256, 2 heads,
    GELU ffn 512): block 0 INT8 ConvRot, block 1 NVFP4, condition_proj INT8."""
    g = torch.Generator().manual_seed(seed)
    model = _step(depth)
    dense, quant = {}, {}
    for name, p in model.state_dict().items():
        prefix, leaf = name.rsplit(".", 1)
        mod = model.get_submodule(prefix)
        if type(mod).__name__ == "QuantLinear":
            if leaf == "weight":
                w = torch.randn(mod.out_features, mod.in_features, generator=g) * 0.02
                if prefix == "condition_proj":
                    quant[prefix] = _int8(w, convrot=False)
                elif prefix.startswith("blocks.0."):
                    quant[prefix] = _int8(w, convrot=True)
                else:
                    quant[prefix] = _nvfp4(w)
            continue
        dense[name] = (1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(p.dtype)
    return dense, quant


def test_comfy_quant_meta_round_trip():
    from minixmax_h3_b200 import checkpoint as ck

    meta = {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256}
    blob = ck.encode_comfy_quant(meta)
    assert blob.dtype == torch.uint8 and blob.dim() == 1
    assert ck.decode_comfy_quant(blob) == meta
    # the reference's decoder reads the same bytes (modules/linear.py:243-245)
    import json
    assert json.loads(bytes(blob.numpy().tobytes()).decode("utf-8")) == meta


def test_load_dit_step(tmp_path):
    from minixmax_h3_b200 import checkpoint as ck

    dense, quant = _synthetic()
    path = tmp_path / "dit.safetensors"
    ck.save_checkpoint(path, dense, quant)
    tensors, metas = ck.load_comfy_tensors(path)
    assert set(metas) == set(quant) and all(metas[k] == quant[k]["meta"] for k in quant)

    model = _step()
    missing, unexpected = ck.load_checkpoint(model, path)
    assert missing == [] and unexpected == []
    for prefix, d in quant.items():
        ql = model.get_submodule(prefix)
        assert ql.quant_format == d["meta"]["format"]
        assert ql.convrot == bool(d["meta"].get("convrot", False))
        if ql.quant_format == "int8_tensorwise":
            assert torch.equal(ql.weight_i8, d["weight"]) and torch.equal(ql.weight_scale, d["weight_scale"])
        else:
            assert torch.equal(ql.weight_u8, d["weight"])
            assert torch.equal(ql.weight_scale, d["weight_scale"].view(torch.uint8).reshape(-1))
            assert torch.equal(ql.weight_scale_2, d["weight_scale_2"].float().reshape(1))
    for name, v in dense.items():
        assert torch.equal(model.state_dict()[name], v), name
    # export -> the same tensors
    dense2, quant2 = ck.export_checkpoint(model)
    assert set(dense2) == set(dense) and all(torch.equal(dense2[k], dense[k]) for k in dense)
    assert set(quant2) == set(quant)
    for prefix, d in quant.items():
        assert quant2[prefix]["meta"] == d["meta"]
        assert torch.equal(quant2[prefix]["weight"], d["weight"])


def test_pre_quant_scale_round_trip(tmp_path):
    """A per-input-channel pre_quant_scale stored beside a quantised weight
    (load/safetensors_quant.py:65-78 passes it to set_quant) is adopted by
    that layer only, and exported again."""
    from minixmax_h3_b200 import checkpoint as ck

    dense, quant = _synthetic()
    g = torch.Generator().manual_seed(5)
    scaled = {"blocks.0.mlp.fc2": 512, "blocks.1.attn.out_proj": 256}  # INT8 ConvRot, NVFP4
    for prefix, k in scaled.items():
        quant[prefix]["pre_quant_scale"] = 0.5 + torch.rand(k, generator=g)
    path = tmp_path / "pqs.safetensors"
    ck.save_checkpoint(path, dense, quant)
    model = _step()
    missing, unexpected = ck.load_checkpoint(model, path)
    assert missing == [] and unexpected == []
    for prefix in quant:
        got = model.get_submodule(prefix).pre_quant_scale
        if prefix in scaled:
            assert torch.equal(got, quant[prefix]["pre_quant_scale"])
        else:
            assert got is None, prefix
    _, quant2 = ck.export_checkpoint(model)
    for prefix in scaled:
        assert torch.equal(quant2[prefix]["pre_quant_scale"], quant[prefix]["pre_quant_scale"])
    assert all("pre_quant_scale" not in quant2[p] for p in quant if p not in scaled)


def test_load_single_linear(tmp_path):
    """load_nvfp4_linear_smoke (load/safetensors_quant.py:218-240): one layer
    of a file, any format, with its optional tensors; unknown prefixes raise."""
    from minixmax_h3_b200 import checkpoint as ck

    dense, quant = _synthetic()
    quant["blocks.1.mlp.fc1"]["pre_quant_scale"] = torch.full((256,), 0.75)
    path = tmp_path / "dit.safetensors"
    ck.save_checkpoint(path, dense, quant)
    nv = ck.load_nvfp4_linear_smoke(path, "blocks.1.mlp.fc1", device="cpu")
    assert nv.quant_format == "nvfp4" and (nv.out_features, nv.in_features) == (512, 256)
    assert torch.equal(nv.weight_u8, quant["blocks.1.mlp.fc1"]["weight"])
    assert torch.equal(nv.pre_quant_scale, quant["blocks.1.mlp.fc1"]["pre_quant_scale"])
    i8 = ck.load_nvfp4_linear_smoke(path, "blocks.0.attn.qkv_proj", device="cpu")
    assert i8.quant_format == "int8_tensorwise" and i8.convrot and i8.pre_quant_scale is None
    assert torch.equal(i8.weight_i8, quant["blocks.0.attn.qkv_proj"]["weight"])
    with pytest.raises(KeyError):
        ck.load_nvfp4_linear_smoke(path, "blocks.0.norm1", device="cpu")


def test_load_one_block_by_prefix_and_wrapper(tmp_path):
    from minixmax_h3_b200 import checkpoint as ck
    from minixmax_h3_b200.block import DiTBlock

    dense, quant = _synthetic()
    wrap = "model.diffusion_model."
    path = tmp_path / "wrapped.safetensors"
    ck.save_checkpoint(path, {wrap + k: v for k, v in dense.items()}, {wrap + k: v for k, v in quant.items()})
    blk = DiTBlock(256, 2, 128, 512, 256, 1e-6, 1e-6, dtype=torch.bfloat16, device="cpu", mlp_act="gelu")
    missing, unexpected = ck.load_checkpoint(blk, path, prefix=wrap + "blocks.1.")
    assert missing == [] and unexpected == []
    assert blk.attn.qkv_proj.quant_format == "nvfp4"
    assert torch.equal(blk.mlp.fc2.weight_u8, quant["blocks.1.mlp.fc2"]["weight"])
    assert torch.equal(blk.norm2.weight, dense["blocks.1.norm2.weight"])


def test_unknown_module_and_bad_scales(tmp_path):
    from minixmax_h3_b200 import checkpoint as ck

    dense, quant = _synthetic(depth=2)
    extra = dict(quant)
    extra["blocks.5.attn.qkv_proj"] = quant["blocks.1.attn.qkv_proj"]
    path = tmp_path / "extra.safetensors"
    ck.save_checkpoint(path, dense, extra)
    with pytest.raises(KeyError):
        ck.load_checkpoint(_step(2), path)
    bad = dict(quant)
    d = dict(quant["blocks.1.mlp.fc1"])
    d["weight_scale"] = d["weight_scale"][:-16]
    bad["blocks.1.mlp.fc1"] = d
    path2 = tmp_path / "bad.safetensors"
    ck.save_checkpoint(path2, dense, bad)
    with pytest.raises(ValueError):
        ck.load_checkpoint(_step(2), path2)
