"""ctypes binding of the in-tree C-ABI library ``libsa3b200.so``.

The library is the only compute path: there is no CPU or PyTorch fallback.
Loading fails with a RuntimeError if the library is missing or lacks a
symbol declared in ``include/sa3b200.h``.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

c_int = ctypes.c_int
c_ll = ctypes.c_longlong
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

SA3_OK = 0
STATUS_NAMES = {
    -1: "SA3_ERR_ARG (bad size / null pointer / inconsistent arguments)",
    -2: "SA3_ERR_ALIGN (pointer or stride violates the 16-byte rule)",
    -3: "SA3_ERR_DTYPE (dtype combination not supported)",
    -4: "SA3_ERR_LAUNCH (CUDA launch or driver call failed)",
    -5: "SA3_ERR_UNSUPPORTED (shape outside what the kernels implement)",
}

DT_BF16, DT_F16, DT_E4M3, DT_F32 = 0, 1, 2, 3
EPI_STORE, EPI_SILU, EPI_SWIGLU, EPI_GATED_RESIDUAL, EPI_RESIDUAL, EPI_QK_NORM = 0, 1, 2, 3, 4, 5
NORM_WRITE, NORM_AMAX = 0, 1


class Epilogue(ctypes.Structure):
    """Mirror of ``sa3_epilogue`` (include/sa3b200.h)."""

    _fields_ = [
        ("kind", c_int),
        ("bias", c_vp),
        ("residual", c_vp),
        ("ld_residual", c_ll),
        ("gate", c_vp),
        ("ld_gate", c_ll),
        ("rows_per_batch", c_int),
        ("row_batch", c_vp),
        ("amax_out", c_vp),
        ("seg_in", c_int),
        ("seg_out", c_int),
        ("seg_offset", c_int),
        ("c_f32", c_int),
        ("qk_gamma", c_vp * 8),
        ("qk_group_width", c_int),
        ("qk_rope_mask", ctypes.c_uint),
        ("qk_eps", c_float),
        ("cos_sin", c_vp),
        ("max_pos", c_int),
        ("row_pos", c_vp),
        ("out_row_map", c_vp),
        ("qk_gamma_table", c_vp),
        ("qk_table_groups", c_int),
        ("c_f16", c_int),
    ]


# name -> argtypes, in the order of include/sa3b200.h
SIGNATURES = {
    "sa3_version": [],
    "sa3_get_device_error": [ctypes.POINTER(c_int)],
    "sa3_gemm": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_ll, c_ll, c_ll, c_int, c_vp, c_vp,
                 ctypes.POINTER(Epilogue), c_vp],
    "sa3_gptq_gemm": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_ll, c_ll, c_int, ctypes.POINTER(Epilogue), c_vp],
    "sa3_gptq_dequant": [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp],
    "sa3_gptq_dequant_orig": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_ll, c_int, c_vp],
    "sa3_permute_cols": [c_vp, c_vp, c_vp, c_int, c_int, c_ll, c_ll, c_vp],
    "sa3_rmsnorm_modulate": [c_vp, c_int, c_vp, c_int, c_int, c_ll, c_ll, c_vp, c_float, c_vp, c_ll, c_int, c_int,
                             c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp],
    "sa3_rmsnorm_quant_fused": [c_vp, c_int, c_vp, c_int, c_int, c_ll, c_ll, c_vp, c_float, c_vp, c_ll, c_int, c_int,
                                c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp],
    "sa3_convert": [c_vp, c_int, c_vp, c_int, c_int, c_int, c_ll, c_ll, c_vp, c_vp],
    "sa3_quantize_e4m3": [c_vp, c_vp, c_int, c_int, c_ll, c_ll, c_vp, c_vp, c_vp, c_vp],
    "sa3_qk_norm_rope": [c_vp, c_int, c_ll, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_vp),
                         ctypes.POINTER(c_int), c_float, c_vp, c_int, c_int, c_vp, c_vp],
    "sa3_attention": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                      c_int, c_int, c_ll, c_ll, c_ll, c_ll, c_int, c_int, c_float, c_int, c_vp, c_vp],
    "sa3_diff_attn_swa": [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp],
    "sa3_fp8_linear_noalloc": [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_ll, c_ll, c_ll, c_vp],
    "sa3_peer_box_bytes": [],
    "sa3_peer_box_alloc": [ctypes.POINTER(c_vp)],
    "sa3_peer_box_free": [c_vp],
    "sa3_ipc_handle_bytes": [],
    "sa3_ipc_get_handle": [c_vp, c_vp],
    "sa3_ipc_open_handle": [c_vp, ctypes.POINTER(c_vp)],
    "sa3_ipc_close_handle": [c_vp],
    "sa3_peer_max": [c_vp, ctypes.POINTER(c_vp), c_int, c_int, c_vp],
}

_lib = None
_lock = threading.Lock()


def library_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libsa3b200.so (building it in-tree first if it is absent)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(f"libsa3b200.so not found at {path}; run the build first")
            _build.build()
        lib = ctypes.CDLL(path)
        for name, argtypes in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as e:
                raise RuntimeError(f"{path} does not export {name}") from e
            fn.argtypes = argtypes
            fn.restype = c_int
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != SA3_OK:
        raise RuntimeError(f"{what} failed: {STATUS_NAMES.get(rc, rc)}")


def device_error() -> int:
    """Read and clear the device error word (synchronises the device)."""
    v = c_int(0)
    check(load().sa3_get_device_error(ctypes.byref(v)), "sa3_get_device_error")
    return v.value
