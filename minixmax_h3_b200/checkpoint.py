"""Comfy-quant safetensors checkpoints -> this package's DiT modules.

The reference ships its DiT as one safetensors file in the Comfy "quant"
convention (load/safetensors_quant.py:25-96): every quantised linear
``<prefix>`` stores

    <prefix>.weight          int8 [N, K]  (int8_tensorwise) or
                             uint8 [N, K/2] e2m1 codes, even element in the
                             high nibble (nvfp4)
    <prefix>.weight_scale    fp32 [N] per-output-channel (int8_tensorwise) or
                             e4m3 block scales in the 128x4 blocked layout (nvfp4)
    <prefix>.weight_scale_2  fp32 per-tensor scale (nvfp4)
    <prefix>.bias, <prefix>.pre_quant_scale   optional
    <prefix>.comfy_quant     uint8 bytes of a JSON object: {"format": ...,
                             "convrot": bool, "convrot_groupsize": int}

and every other tensor (norm weights, the adaLN projection when it is dense)
is a plain state-dict entry.  Module prefixes are paths from the DiT root
(``blocks.3.attn.qkv_proj``, ``condition_proj``, ...); this package's
``DiTStep`` / ``DiTBlock`` use the reference's attribute names
(model/dit.py:156-167, 291-296, 304-329, 400-433, 668-690), so keys map one
to one.  Quantised tensors are adopted as stored by ``QuantLinear.set_quant``
(the same call the reference makes, modules/linear.py:105-169); the device
repack (NVFP4 nibble order) happens once on first use.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Optional

import torch
import torch.nn as nn

from .modules import Linear, QuantLinear, decode_comfy_quant

COMFY_QUANT_SUFFIX = ".comfy_quant"


def encode_comfy_quant(meta: dict[str, Any]) -> torch.Tensor:
    """Inverse of ``decode_comfy_quant``: the uint8 tensor a checkpoint stores."""
    raw = json.dumps(meta, sort_keys=True).encode("utf-8")
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone()


def load_comfy_tensors(path: str | Path) -> tuple[dict[str, torch.Tensor], dict[str, dict[str, Any]]]:
    """All tensors of a safetensors file plus the decoded quant metadata per
    module prefix (load/safetensors_quant.py:25-37)."""
    from safetensors import safe_open

    tensors: dict[str, torch.Tensor] = {}
    metas: dict[str, dict[str, Any]] = {}
    with safe_open(str(path), framework="pt") as f:
        for key in f.keys():
            if key.endswith(COMFY_QUANT_SUFFIX):
                metas[key[: -len(COMFY_QUANT_SUFFIX)].rstrip(".")] = decode_comfy_quant(f.get_tensor(key))
            else:
                tensors[key] = f.get_tensor(key)
    return tensors, metas


def select_prefix(tensors: dict[str, torch.Tensor], metas: dict[str, dict[str, Any]], prefix: str
                  ) -> tuple[dict[str, torch.Tensor], dict[str, dict[str, Any]]]:
    """Keep the keys under ``prefix`` with the prefix removed: a wrapper
    (``model.diffusion_model.``) or one block of a full model (``blocks.3.``)."""
    if not prefix:
        return tensors, metas
    n = len(prefix)
    return ({k[n:]: v for k, v in tensors.items() if k.startswith(prefix)},
            {k[n:]: v for k, v in metas.items() if k.startswith(prefix)})


def _resolve_module(root: nn.Module, dotted: str) -> tuple[nn.Module, str]:
    parent = root
    parts = dotted.split(".")
    for p in parts[:-1]:
        parent = getattr(parent, p)
    return parent, parts[-1]


def apply_quant_modules(model: nn.Module, tensors: dict[str, torch.Tensor], metas: dict[str, dict[str, Any]], *,
                        device: Optional[torch.device] = None, compute_dtype: torch.dtype = torch.bfloat16
                        ) -> dict[str, torch.Tensor]:
    """Replace every linear covered by quant metadata with a ``QuantLinear``
    holding the checkpoint's tensors; return the remaining dense entries
    (load/safetensors_quant.py:40-96).  Prefixes naming no module of
    ``model`` raise ``KeyError``; non-linear targets (the text encoder's
    embedding, which is not on this path) are left to the dense remainder."""
    consumed: set[str] = set()
    for prefix, meta in sorted(metas.items()):
        w_key = f"{prefix}.weight"
        if w_key not in tensors:
            continue
        try:
            parent, attr = _resolve_module(model, prefix)
            child = getattr(parent, attr)
        except AttributeError as e:
            raise KeyError(f"checkpoint module {prefix!r} has no counterpart in {type(model).__name__}") from e
        if not isinstance(child, (Linear, QuantLinear, nn.Linear)):
            continue
        ql = QuantLinear.from_quant_tensors(
            tensors[w_key], meta=meta, weight_scale=tensors.get(f"{prefix}.weight_scale"),
            weight_scale_2=tensors.get(f"{prefix}.weight_scale_2"), bias=tensors.get(f"{prefix}.bias"),
            pre_quant_scale=tensors.get(f"{prefix}.pre_quant_scale"), device=device, compute_dtype=compute_dtype)
        setattr(parent, attr, ql)
        consumed.update({w_key, f"{prefix}.weight_scale", f"{prefix}.weight_scale_2", f"{prefix}.bias",
                         f"{prefix}.pre_quant_scale"})
    return {k: v for k, v in tensors.items() if k not in consumed}


def load_checkpoint(model: nn.Module, path: str | Path, *, device: Optional[torch.device] = None,
                    prefix: str = "", compute_dtype: torch.dtype = torch.bfloat16) -> tuple[list[str], list[str]]:
    """Load a Comfy-quant safetensors file into ``model`` (a ``DiTStep``, or a
    ``DiTBlock`` with ``prefix="blocks.<i>."``): quantised linears through
    ``apply_quant_modules``, everything else with ``load_state_dict``
    (load/safetensors_quant.py:99-146).  Returns (missing, unexpected) dense
    keys, ignoring the quantised projections' empty ``weight`` shells the way
    the reference does."""
    tensors, metas = select_prefix(*load_comfy_tensors(path), prefix)
    remaining = apply_quant_modules(model, tensors, metas, device=device, compute_dtype=compute_dtype)
    missing, unexpected = model.load_state_dict(remaining, strict=False)
    quant_prefixes = {name for name, m in model.named_modules() if isinstance(m, QuantLinear)}
    missing = [m for m in missing if m.rsplit(".", 1)[0] not in quant_prefixes]
    return missing, list(unexpected)


def load_nvfp4_linear_smoke(path: str | Path, layer_prefix: str = "model.layers.0.mlp.gate_proj", *,
                            device: Optional[torch.device] = None,
                            dtype: torch.dtype = torch.bfloat16) -> QuantLinear:
    """One quantised linear of a checkpoint as a ``QuantLinear``
    (load/safetensors_quant.py:218-240, same name and arguments): whatever
    format its metadata names, with its scales, bias and pre_quant_scale.
    Raises ``KeyError`` when the file has no quant metadata for the prefix."""
    tensors, metas = load_comfy_tensors(path)
    if layer_prefix not in metas:
        raise KeyError(f"{layer_prefix} not in quant metas")
    return QuantLinear.from_quant_tensors(
        tensors[f"{layer_prefix}.weight"], meta=metas[layer_prefix],
        weight_scale=tensors.get(f"{layer_prefix}.weight_scale"),
        weight_scale_2=tensors.get(f"{layer_prefix}.weight_scale_2"), bias=tensors.get(f"{layer_prefix}.bias"),
        pre_quant_scale=tensors.get(f"{layer_prefix}.pre_quant_scale"), device=device, compute_dtype=dtype)


def save_checkpoint(path: str | Path, dense: dict[str, torch.Tensor],
                    quant: dict[str, dict[str, Any]]) -> None:
    """Write a Comfy-quant safetensors file: ``dense`` state-dict entries plus,
    per module prefix, a dict with ``weight``, ``weight_scale``, optional
    ``weight_scale_2`` / ``bias`` / ``pre_quant_scale`` and ``meta`` (the
    layout ``load_comfy_tensors`` reads)."""
    from safetensors.torch import save_file

    # own copies: safetensors refuses entries that share storage
    out = {k: v.detach().cpu().clone() for k, v in dense.items()}
    for prefix, d in quant.items():
        for name in ("weight", "weight_scale", "weight_scale_2", "bias", "pre_quant_scale"):
            if d.get(name) is not None:
                out[f"{prefix}.{name}"] = d[name].detach().cpu().clone()
        out[f"{prefix}{COMFY_QUANT_SUFFIX}"] = encode_comfy_quant(d["meta"])
    save_file(out, str(path))


def export_checkpoint(model: nn.Module) -> tuple[dict[str, torch.Tensor], dict[str, dict[str, Any]]]:
    """(dense, quant) of a model in the layout ``save_checkpoint`` writes:
    every ``QuantLinear`` as its checkpoint tensors (INT8 codes + per-channel
    scales, or NVFP4 hi-first codes + blocked scales + per-tensor scale) and
    metadata, everything else as state-dict entries.  Weights already
    reordered for the fused SwiGLU epilogue are refused (export before the
    first forward)."""
    quant: dict[str, dict[str, Any]] = {}
    quant_prefixes = set()
    for name, m in model.named_modules():
        if not isinstance(m, QuantLinear) or m.quant_format is None:
            continue
        if m._row_perm is not None:
            raise ValueError(f"{name}: weights are in the SwiGLU-interleaved order; export before running forward")
        meta: dict[str, Any] = {"format": m.quant_format}
        if m.convrot:
            meta.update(convrot=True, convrot_groupsize=m.group_size)
        if m.quant_format == "int8_tensorwise":
            d = {"weight": m.weight_i8, "weight_scale": m.weight_scale}
        else:
            d = {"weight": m.weight_u8, "weight_scale": m.weight_scale, "weight_scale_2": m.weight_scale_2}
        if m.bias is not None and m.bias.numel():
            d["bias"] = m.bias.data
        if m.pre_quant_scale is not None:
            d["pre_quant_scale"] = m.pre_quant_scale
        d["meta"] = meta
        quant[name] = d
        quant_prefixes.add(name)
    dense = {k: v for k, v in model.state_dict().items() if k.rsplit(".", 1)[0] not in quant_prefixes}
    return dense, quant
