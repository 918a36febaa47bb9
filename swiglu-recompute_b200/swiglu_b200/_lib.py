"""ctypes binding of libswiglu_b200.so (the C ABI of include/swiglu_b200.h).

There is no fallback: if the library is missing the first call raises, so a
machine without the native build can never silently run another code path.
"""
from __future__ import annotations

import ctypes
import os
import re

from .build import INCLUDE_DIR, LIB_PATH

# Mirrors of the header's enums.
OK = 0
F32, BF16 = 0, 1
LAYOUT_STD, LAYOUT_PACKED128 = 0, 1
W1_ROWS, W1_T = 0, 1

HEADER = os.path.join(INCLUDE_DIR, "swiglu_b200.h")

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int

# name -> argtypes; restype is int unless listed in _RESTYPES.
_SIGNATURES = {
    "swiglu_b200_abi_version": [],
    "swiglu_b200_status_string": [_i],
    "swiglu_b200_last_error_message": [],
    "swiglu_b200_device_status": [ctypes.POINTER(ctypes.c_uint32), _i],
    "swiglu_b200_set_gemm_path": [_i],
    "swiglu_b200_set_sm_reserve": [_i],
    "swiglu_b200_gemm_plan": [_i64, _i64, _i, _i, ctypes.POINTER(_i)],
    "swiglu_b200_swiglu_fwd_plan": [_i64, _i64, _i64, _i, ctypes.POINTER(_i)],
    "swiglu_b200_set_stream_workspace": [_p, ctypes.c_size_t, _p],
    "swiglu_b200_fused_matmul_swiglu_save_preact":
        [_p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _p],
    "swiglu_b200_matmul": [_p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _p],
    "swiglu_b200_matmul_tiled": [_p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _p],
    "swiglu_b200_matmul_scatter_rows":
        [_p, _p, _i64, _i64, _i64, _i, _i, _i, ctypes.POINTER(_p), _i, _i, _i64, _p],
    "swiglu_b200_tp_signal": [ctypes.POINTER(_p), _i, _i, ctypes.c_uint32, _p],
    "swiglu_b200_tp_reduce_rows": [_p, _p, _i, ctypes.c_uint32, _p, _i64, _i64, _i, _p],
    "swiglu_b200_matmul_reduce_rows_noalloc": [_p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _p],
    "swiglu_b200_bwd_dw2": [_p, _p, _p, _i64, _i64, _i64, _i, _i, _p],
    "swiglu_b200_bwd_grad_preact_inplace": [_p, _p, _p, _i64, _i64, _i64, _i, _i, _p],
    "swiglu_b200_bwd_grad_preact_inplace_emit_h": [_p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _p],
    "swiglu_b200_forward_logic": [_p, _p, _i64, _i64, _i, _i, _p],
    "swiglu_b200_backward_logic": [_p, _p, _p, _i64, _i64, _i, _i, _p],
    "swiglu_b200_pack_weight_chunked": [_p, _p, _i64, _i64, _i64, _i, _i, _p],
    "swiglu_b200_quantize_rows_e4m3": [_p, _p, _p, _i64, _i64, _i, _p],
    "swiglu_b200_fused_matmul_swiglu_e4m3": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _p],
    "swiglu_b200_matmul_e4m3": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _p],
    "swiglu_b200_mlp_forward":
        [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _i, _i, _i, _p],
    "swiglu_b200_mlp_backward":
        [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _i, _i, _p],
}
_RESTYPES = {
    "swiglu_b200_status_string": ctypes.c_char_p,
    "swiglu_b200_last_error_message": ctypes.c_char_p,
}


class SwigluError(RuntimeError):
    """A non-zero status from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_LIB: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(swiglu_b200_\w+)\s*\(", text)))


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m swiglu_b200.build` "
            "(from swiglu-recompute_b200/) or __graft_entry__.build(). "
            "There is no non-native fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    if lib.swiglu_b200_abi_version() != 1:
        raise ImportError("libswiglu_b200.so ABI version mismatch")
    _LIB = lib
    return lib


def check(status: int) -> None:
    if status != OK:
        lib = load()
        name = lib.swiglu_b200_status_string(status).decode()
        detail = lib.swiglu_b200_last_error_message().decode()
        raise SwigluError(status, f"{name}: {detail}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def set_gemm_path(mode: int) -> None:
    """0 = by size, 1 = single-SM tcgen05 kernel, 2 = 2-SM (CTA pair) kernel with 256 x 256
    tiles, 3 = 2-SM kernel with 256 x 512 tiles."""
    call("swiglu_b200_set_gemm_path", int(mode))


def set_sm_reserve(sms: int) -> None:
    """SMs the persistent GEMM launches leave free for other streams' kernels
    (process-wide; 0 = use every SM)."""
    call("swiglu_b200_set_sm_reserve", int(sms))


def gemm_plan(M: int, N: int, tile_n: int = 0, num_sms: int = 148) -> int:
    """Kernel family of a bf16 GEMM with an [M, N] output: 1 = single-SM,
    2 = CTA pair 256 x 256 tiles, 3 = CTA pair 256 x 512 tiles (host-only)."""
    fam = ctypes.c_int(0)
    call("swiglu_b200_gemm_plan", int(M), int(N), int(tile_n), int(num_sms), ctypes.byref(fam))
    return int(fam.value)


def swiglu_fwd_plan(M: int, K: int, H: int, num_sms: int = 148) -> int:
    """Kernel family of the bf16 GEMM1 + SwiGLU forward at M tokens, K inputs
    and H hidden units (same codes as gemm_plan; host-only)."""
    fam = ctypes.c_int(0)
    call("swiglu_b200_swiglu_fwd_plan", int(M), int(K), int(H), int(num_sms), ctypes.byref(fam))
    return int(fam.value)


def device_status(clear: bool = True) -> int:
    """Timeout bits of the current device's kernels (0 = healthy); synchronises."""
    bits = ctypes.c_uint32(0)
    load().swiglu_b200_device_status(ctypes.byref(bits), 1 if clear else 0)
    return int(bits.value)
