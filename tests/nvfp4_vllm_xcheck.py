"""Cross-check of the oracle's NVFP4 quantiser against an independent
implementation: vllm's pure-torch ``ref_nvfp4_quant``
(vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py,
vllm 0.22).  Run as a child process by ``test_oracle_pins.py`` so that vllm's
import-time configuration stays out of the test process; prints one JSON
object.

The two restate the same published recipe in different fp32 orders: the
oracle divides (s = e4m3(amax_b / (6 gs)), q = e2m1(x / (s gs)), gs =
amax / 2688), vllm multiplies by reciprocals (s = e4m3(g * amax_b / 6),
q = e2m1(x * 1/(s/g)), g = 2688 / amax).  Both round half to even.  For
every block scale and code on which they disagree, this reports how far the
exact (fp64) value lies from the rounding midpoint between the two results;
0 means an exact tie, decided by each recipe's own fp32 roundings.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import h3_oracle as O  # noqa: E402

E2M1_MIDPOINTS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=torch.float64)


def compare(x: torch.Tensor, ref_nvfp4_quant) -> dict:
    xb = x.to(torch.bfloat16)
    m, k = xb.shape
    amax = xb.float().abs().max()
    mine = O.nvfp4_quantize(xb, hi_first=True)
    vals, scale = ref_nvfp4_quant(xb.float(), (torch.tensor(2688.0) / amax).float().reshape(1), 16)

    my_sf = torch.from_numpy(O.from_blocked(mine["sf"].numpy(), m, k // 16)).int()
    v_sf = scale.to(torch.float8_e4m3fn).view(torch.uint8).int()
    sf_bad = v_sf != my_sf
    amax_b = xb.double().abs().reshape(m, k // 16, 16).amax(-1)
    exact_s = amax_b * 448.0 / amax.double()
    lo = torch.from_numpy(O.e4m3_decode(torch.minimum(my_sf, v_sf).numpy().astype(np.uint8))).double()
    hi = torch.from_numpy(O.e4m3_decode(torch.maximum(my_sf, v_sf).numpy().astype(np.uint8))).double()
    sf_tie_dist = ((exact_s - (lo + hi) / 2).abs() / ((lo + hi) / 2))[sf_bad]

    s = torch.from_numpy(O.e4m3_decode(my_sf.numpy().astype(np.uint8))).double().repeat_interleave(16, 1)
    my_vals = O.nvfp4_dequantize(mine["codes"], torch.ones(1), mine["sf"], k, True).double()
    my_e2m1 = torch.where(s > 0, my_vals / s.clamp(min=1e-300), torch.zeros_like(my_vals))
    code_bad = (my_e2m1 != vals.double()) & ~sf_bad.repeat_interleave(16, 1)
    exact_q = (xb.double() * 2688.0 / (s * amax.double())).abs()[code_bad]
    code_tie_dist = (exact_q[:, None] - E2M1_MIDPOINTS[None]).abs().min(1).values

    return {
        "scales": int(my_sf.numel()),
        "scale_mismatches": int(sf_bad.sum()),
        "scale_steps_apart_max": int((my_sf - v_sf).abs().max()),
        "scale_tie_dist_max": float(sf_tie_dist.max()) if sf_bad.any() else 0.0,
        "codes_compared": int((~sf_bad).sum()) * 16,
        "code_mismatches": int(code_bad.sum()),
        "code_tie_dist_max": float(code_tie_dist.max()) if code_bad.any() else 0.0,
    }


def main() -> None:
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import ref_nvfp4_quant

    g = torch.Generator().manual_seed(0)
    acts = torch.where(torch.rand(1024, 3072, generator=g) < 0.001, 20, 1) * torch.randn(1024, 3072, generator=g)
    wts = torch.randn(3072, 3072, generator=g) * 0.02
    # a global max of 57/512: block maxima with the factor 57 in their
    # mantissa then put the exact scale ratio on e4m3 midpoints (about 1 %)
    wts[0, 0] = 0.111328125
    print(json.dumps({"activations": compare(acts, ref_nvfp4_quant), "weights": compare(wts, ref_nvfp4_quant)}))


if __name__ == "__main__":
    main()
