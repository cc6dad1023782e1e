"""ctypes binding of ``libh3b.so`` (declared in ``include/h3b.h``).

The library is the only compute path: if it is missing or fails to load, every
op raises instead of falling back to PyTorch or the CPU.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libh3b.so")

c_ptr = ctypes.c_void_p
c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_f32 = ctypes.c_float

# name -> argument types, in the order of include/h3b.h
SIGNATURES: dict[str, list] = {
    "h3b_version": [],
    "h3b_device_status": [c_ptr, c_int],
    "h3b_quant_i8_rows": [c_ptr, c_int, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr],
    "h3b_quant_i8_rows_convrot": [c_ptr, c_int, c_i64, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr],
    "h3b_gemm_i8_bf16": [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_int,
                         c_i64, c_i64, c_i64, c_ptr],
    "h3b_gemm_i8_acc_i32": [c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_i64, c_ptr],
    "h3b_amax_bf16": [c_ptr, c_i64, c_ptr, c_ptr],
    "h3b_quant_nvfp4": [c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_int, c_ptr],
    "h3b_quant_nvfp4_gelu": [c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_int, c_ptr],
    "h3b_gelu_amax_scan": [c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr],
    "h3b_nvfp4_swap_nibbles": [c_ptr, c_ptr, c_i64, c_ptr],
    "h3b_gemm_nvfp4_bf16": [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64,
                            c_ptr, c_ptr, c_int, c_i64, c_i64, c_i64, c_ptr],
    "h3b_attention_fwd": [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                          c_i64, c_i64, c_f32, c_ptr],
    "h3b_ipc_export": [c_ptr, c_ptr, c_ptr],
    "h3b_ipc_import": [c_ptr, c_i64, c_ptr],
    "h3b_ipc_close": [c_ptr, c_i64],
    "h3b_gemm_i8_seq2head": [c_ptr] * 6 + [c_i64] * 6 + [c_ptr],
    "h3b_gemm_nvfp4_seq2head": [c_ptr] * 8 + [c_i64] * 6 + [c_ptr],
    "h3b_attention_fwd_head2seq": [c_ptr] * 4 + [c_i64] * 5 + [c_ptr] + [c_i64] * 7 + [c_f32, c_ptr],
    "h3b_qk_rmsnorm_rope": [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_f32, c_ptr, c_i64, c_ptr,
                            c_int, c_int, c_ptr],
    "h3b_rmsnorm_modulate": [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_f32, c_ptr,
                             c_ptr],
    "h3b_gate_residual": [c_ptr, c_ptr, c_i64, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_ptr],
    "h3b_rmsnorm_modulate_quant_i8": [c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_f32, c_i64,
                                      c_ptr, c_ptr, c_ptr],
    "h3b_rmsnorm_modulate_quant_nvfp4_noalloc": [c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                                                 c_f32, c_ptr, c_ptr, c_ptr, c_int, c_ptr],
    "h3b_selftest_wait_timeout": [c_ptr] * 7 + [c_i64] * 3 + [c_ptr],
    "h3b_attention_merge_lse": [c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_int, c_ptr, c_ptr, c_ptr],
}

ERRORS = {
    1: "unsupported or inconsistent shape",
    2: "pointer or stride alignment violated",
    3: "unsupported dtype",
    4: "kernel launch failed",
    5: "TMA descriptor rejected",
    6: "bounded device wait timed out",
    7: "device reported a failure",
    8: "bad argument",
}


class H3bError(RuntimeError):
    """Non-zero status from a libh3b entry point."""

    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed with status {code} ({ERRORS.get(code, 'unknown')})")
        self.fn = fn
        self.code = code


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libh3b.so once and declares every exported signature."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m minixmax_h3_b200.build` (no CPU fallback exists)"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            if not hasattr(handle, name):
                continue  # reported by tests/test_abi.py; calling it raises below
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = c_int
        _LIB = handle
    return _LIB


# Entry points that launch no kernel of this library.
_NO_LAUNCH = {"h3b_version", "h3b_device_status"}
LAUNCHES = [0]  # kernels this process has launched through the ABI


def call(name: str, *args) -> None:
    """Calls an entry point and raises H3bError on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise H3bError(name, rc)
    if name not in _NO_LAUNCH:
        LAUNCHES[0] += 1


def device_status(clear: bool = True) -> tuple[int, int, int, int]:
    """(code, site, info, block) of the first device-side error, 0s if none."""
    buf = (ctypes.c_int32 * 4)()
    call("h3b_device_status", ctypes.cast(buf, c_ptr), 1 if clear else 0)
    return tuple(int(v) for v in buf)  # type: ignore[return-value]
