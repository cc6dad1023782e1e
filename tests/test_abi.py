"""CPU: the C-ABI library loads, exports every entry point include/h3b.h
declares, and rejects bad arguments on the host without touching a GPU."""
from __future__ import annotations

import re
from pathlib import Path

import pytest

from minixmax_h3_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "h3b.h"


def declared() -> list[str]:
    return re.findall(r"H3B_API\s+int\s+(h3b_\w+)\s*\(", HEADER.read_text())


def test_header_and_binding_agree():
    names = declared()
    assert len(names) >= 12
    assert sorted(names) == sorted(_lib.SIGNATURES)


def test_binding_argument_counts_match_the_header():
    """Each ctypes signature has as many arguments as the C declaration
    (a wrong count would pass garbage across the ABI without an error)."""
    text = HEADER.read_text()
    found = list(re.finditer(r"H3B_API\s+int\s+(h3b_\w+)\s*\(([^;]*?)\)\s*;", text, re.S))
    assert len(found) == len(declared())
    for m in found:
        name, params = m.group(1), " ".join(m.group(2).split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(_lib.SIGNATURES[name]) == n, (name, n, len(_lib.SIGNATURES[name]))


def test_library_exports_every_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.h3b_version() >= 100


@pytest.mark.parametrize("name,args,code", [
    ("h3b_quant_i8_rows", (None, 0, 4, 64, 64, None, None, None), 8),
    ("h3b_quant_i8_rows_convrot", (16, 0, 4, 3072, 3072, 128, 16, 16, None, None), 1),     # group 128
    ("h3b_quant_i8_rows_convrot", (16, 0, 4, 1000, 1000, 256, 16, 16, None, None), 1),     # k % 256
    ("h3b_quant_i8_rows_convrot", (16, 0, 4, 24576, 24576, 256, 16, 16, None, None), 1),   # k > 12288
    ("h3b_gemm_i8_bf16", (16, 16, 16, 16, None, 16, 64, None, None, 0, None, None, 0, 4, 48, 128, None), 1),  # n%32
    ("h3b_gemm_i8_bf16", (16, 16, 16, 16, None, 16, 64, None, None, 0, None, None, 0, 4, 64, 100, None), 1),  # k%128
    ("h3b_gemm_i8_bf16", (16, 16, 16, 16, None, 16, 64, None, None, 0, None, None, 2, 4, 64, 128, None), 8),  # gate
    ("h3b_gemm_nvfp4_bf16", (16,) * 6 + (None, 16, 256, None, None, 0, None, None, 0, 4, 256, 128, None), 1),
    ("h3b_quant_nvfp4", (16, 4, 48, 48, 16, 16, 16, 16, 1, None), 1),                       # k % 64
    ("h3b_quant_nvfp4_gelu", (None, 4, 64, 64, 16, 16, 16, 16, 0, None), 8),                # null y
    ("h3b_quant_nvfp4_gelu", (16, 4, 48, 48, 16, 16, 16, 16, 0, None), 1),                  # k % 64
    ("h3b_quant_nvfp4_gelu", (16, 0, 64, 64, 16, 16, 16, 16, 0, None), 1),                  # needs a row
    ("h3b_quant_nvfp4_gelu", (16, 4, 64, 64, 16, 16, 18, 16, 0, None), 2),                  # sf unaligned
    ("h3b_gelu_amax_scan", (None, 4, 64, 64, 16, None), 8),                                  # null y
    ("h3b_gelu_amax_scan", (16, 4, 60, 64, 16, None), 1),                                    # k % 8
    ("h3b_gemm_nvfp4_bf16", (16,) * 6 + (None, 16, 256, None, None, 0, None, None, 5, 4, 256, 256, None), 8),  # epi 5
    ("h3b_attention_fwd", (None,) * 6 + (1, 1, 1, 128, 128, 128, 128, 128, 128, 0.1, None), 8),
    ("h3b_attention_fwd", (16,) * 4 + (None, None, 1, 1, 1, 100, 128, 128, 128, 128, 128, 0.1, None), 2),
    ("h3b_rmsnorm_modulate", (16, 16, 4, 100, 100, 16, 16, 16, 0, None, 1e-6, None, None), 1),
    ("h3b_amax_bf16", (16, 7, 16, None), 1),
    ("h3b_attention_merge_lse", (None, 16, 16, 16, 4, 1, 0, None, None, None), 8),                # null acc
    ("h3b_attention_merge_lse", (16, 16, 16, 16, 4, 0, 0, None, None, None), 1),                  # heads 0
    ("h3b_attention_merge_lse", (16, 16, 24, 16, 4, 1, 0, None, None, None), 2),                  # blk unaligned
    ("h3b_rmsnorm_modulate_quant_i8", (16, 4, 3072, 3072, 16, 16, 16, 0, None, 1e-6, 128, 16, 16, None), 1),
    ("h3b_rmsnorm_modulate_quant_i8", (16, 4, 1000, 1000, 16, 16, 16, 0, None, 1e-6, 256, 16, 16, None), 1),
    ("h3b_rmsnorm_modulate_quant_i8", (16, 4, 3072, 3072, 16, 16, 16, 0, None, 1e-6, 0, None, 16, None), 8),
    # allocation-free NVFP4 input: rows beyond its 16 MiB array, and hidden % 64
    ("h3b_rmsnorm_modulate_quant_nvfp4_noalloc", (16, 8193, 1024, 1024, 16, 16, 16, 0, None, 1e-6, 16, 16, 16, 1,
                                                  None), 1),
    ("h3b_rmsnorm_modulate_quant_nvfp4_noalloc", (16, 4, 1000, 1000, 16, 16, 16, 0, None, 1e-6, 16, 16, 16, 1,
                                                  None), 1),
])
def test_host_side_validation(name, args, code):
    fn = getattr(_lib.lib(), name)
    assert fn(*args) == code


@pytest.mark.parametrize("name,args", [
    ("h3b_gemm_i8_bf16", (16, 16, 16, 16, None, 16, 64, None, None, 0, None, None, 0, 0, 64, 128, None)),
    ("h3b_gemm_i8_acc_i32", (16, 16, 16, 0, 64, 128, None)),
    ("h3b_gemm_nvfp4_bf16", (16,) * 6 + (None, 16, 192, None, None, 0, None, None, 0, 0, 192, 256, None)),
    ("h3b_attention_fwd", (16,) * 4 + (None, None, 2, 0, 128, 128, 128, 128, 128, 128, 128, 0.1, None)),
    ("h3b_quant_i8_rows", (16, 0, 0, 64, 64, 16, 16, None)),
    ("h3b_gelu_amax_scan", (16, 0, 64, 64, 16, None)),
    ("h3b_gemm_nvfp4_bf16", (16,) * 6 + (None, 16, 256, None, None, 0, None, None, 4, 0, 256, 256, None)),  # posmax
])
def test_empty_batch_is_a_no_op(name, args):
    """Zero rows: H3B_OK before any launch (the reference returns an empty
    result for an empty batch)."""
    fn = getattr(_lib.lib(), name)
    assert fn(*args) == 0
