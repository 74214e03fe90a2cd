"""Loader of libh3b200.so, the sm_100a kernels behind include/h3b200.h.

There is no fallback: if the library is missing or cannot be loaded, every operator
raises.  The library is built in-tree by minimax-h3-2xt4_b200/build.py (also run by
__graft_entry__.build()).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libh3b200.so"

H3_OK = 0
H3_ERR_INVALID = 1
H3_ERR_CUDA = 2
H3_ERR_TIMEOUT = 3
H3_ERR_UNSUPPORTED = 4

IN_GATEUP_F16 = 0
IN_ACT_F32 = 1
IN_ACT_F16 = 2
DIV_RN = 0
DIV_FAST = 1
OUT_F32 = 0
OUT_F16 = 1
OUT_RESIDUAL = 2
OUT_I32 = 3

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_U32 = ctypes.c_uint32
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "h3_abi_version": [],
    "h3_status_string": [_I],
    "h3_device_error": [_I, _P],
    "h3_device_error_peek": [_I, _P],
    "h3_sm_clock_probe": [ctypes.c_uint64, _P, _P],
    "h3_column_quantize": [_P, _I64, _I64, _I, _P, _P, _P],
    "h3_int8_gemm_i32": [_P, _P, _I64, _I64, _I64, _P, _P],
    "h3_int8_gemm_column": [_P, _P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _P],
    "h3_int8_gemm_swiglu": [_P, _P, _I64, _I64, _I64, _P, _P, _P, _I, _P, _P],
    "h3_column_dequantize": [_P, _I64, _I64, _P, _P, _I64, _P, _P],
    "h3_swiglu_rotate_max": [_P, _I, _I64, _I64, _P, _P, _P],
    "h3_swiglu_rotate_quantize": [_P, _I, _I64, _I64, _P, _I, _P, _P, _P],
    "h3_swiglu_rotate_quantize_local": [_P, _I, _I64, _I64, _I, _P, _P, _P, _P],
    "h3_row_quantize": [_P, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _P],
    "h3_transport_shift": [_I64],
    "h3_int8_gemm_row_encode": [_P, _P, _I64, _I64, _I64, _I, _P, _P],
    "h3_int8_gemm_row_dequant": [_P, _P, _I64, _I64, _I64, _P, _P, _I, _P, _P, _P, _I64, _P, _P],
    "h3_fp16_encode": [_P, _I64, _I, _P, _P],
    "h3_fp16_decode": [_P, _I64, _I, _P, _P],
    "h3_row_reduce_finish": [_P, _I, _I64, _I64, _I64, _I, _P, _P, _I, _P, _P, _P, _I64, _P, _P],
    "h3_dequantize_i32": [_P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _P],
    "h3_gated_add": [_P, _I, _I64, _I64, _P, _P, _I64, _P, _P],
    "h3_int8_gemm_row_pack8": [_P, _P, _I64, _I64, _I64, _P, _P],
    "h3_modulated_norm_quantize": [_P, _I64, _I64, _P, ctypes.c_float, _P, _P, _I64, _P, _I, _P,
                                   _P, _P, _P],
    "h3_pack8": [_P, _I64, _I64, _P, _P],
    "h3_unpack8_finish": [_P, _I, _I64, _I64, _I64, _P, _P, _I, _P, _P, _P, _I64, _P, _P],
    "h3_peer_reduce_int8": [_PP, _I, _I, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P,
                            _U32, _P],
    "h3_peer_reduce": [_PP, _I, _I, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P, _I64, _P,
                       _U32, _P],
    "h3_peer_reduce_pushed": [_PP, _I, _I, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P, _I64, _P,
                       _U32, _P],
    "h3_int8_gemm_row_encode_push": [_P, _P, _I64, _I64, _I64, _I, _PP, _I, _I, _I64, _P],
    "h3_peer_signal": [_PP, _I, _I, _I64, _I, _U32, _I, _P],
    "h3_peer_reduce_staged": [_PP, _I, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P,
                              _I64, _P, _U32, _P],
    "h3_copy_async": [_P, _P, _I64, _P],
    "h3_peer_reduce_nvls": [_PP, _P, _I, _I, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P,
                            _I64, _P, _U32, _P],
    "h3_peer_gather": [_PP, _I, _I, _I64, _I64, _I64, _I64, _P, _U32, _P],
    "h3_swiglu_rotate_quantize_peer": [_P, _I, _I64, _I64, _PP, _I, _I, _I64, _U32, _I, _P, _P,
                                       _P, _P],
    "h3_expf_compare": [_P, _I64, _P, _P, _P],
    "h3_silu_compare": [_P, _I64, _P, _P, _P, _P],
    "h3_quant_compare": [_P, _P, _I64, _P, _P, _P],
    "h3_column_linear_noalloc": [_P, _I64, _I64, _I, _P, _I64, _P, _I64, _P, _P, _P],
    "h3_column_linear_noalloc_error": [_I, _P],
}
_RESTYPES = {"h3_status_string": ctypes.c_char_p}

_lib = None


class H3Error(RuntimeError):
    """A CUDA-side failure of the native library (launch error or timeout)."""


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it on first use.  Raises when absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("H3B200_LIB", str(LIB_PATH)))
    if not path.exists():
        raise ImportError(
            f"libh3b200.so not found at {path}; build it with "
            "`python minimax-h3-2xt4_b200/build.py` (the INT8 path has no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, _I)
    if lib.h3_abi_version() != 1:
        raise ImportError("libh3b200.so ABI version mismatch")
    _lib = lib
    return lib


def check(status: int, name: str) -> None:
    """Maps a C status to the exception the reference raises for the same case."""
    if status == H3_OK:
        return
    msg = load().h3_status_string(status).decode()
    if status in (H3_ERR_INVALID, H3_ERR_UNSUPPORTED):
        raise ValueError(f"{name}: {msg}")
    raise H3Error(f"{name}: {msg}")


# Entry points that enqueue exactly one kernel per successful call.
_LAUNCHING = {n for n in SIGNATURES if n not in (
    "h3_abi_version", "h3_status_string", "h3_device_error", "h3_device_error_peek",
    "h3_transport_shift", "h3_column_linear_noalloc_error", "h3_sm_clock_probe",
    "h3_copy_async")}
_launches = 0


def call(name: str, *args) -> None:
    global _launches
    check(getattr(load(), name)(*args), name)
    if name in _LAUNCHING:
        _launches += 1


def launch_count() -> int:
    """Number of native kernels this process has enqueued through call()."""
    return _launches


def device_error(device: int) -> int:
    """Reads and clears the device-side error word (0 when nothing failed)."""
    code = ctypes.c_int(0)
    check(load().h3_device_error(int(device), ctypes.byref(code)), "h3_device_error")
    return code.value


def device_error_peek(device: int) -> int:
    """The device-side error word as it stands, read from host-mapped memory without
    synchronising or clearing it (0 when nothing failed so far)."""
    code = ctypes.c_int(0)
    check(load().h3_device_error_peek(int(device), ctypes.byref(code)), "h3_device_error_peek")
    return code.value


def raise_on_device_error(device: int, where: str) -> None:
    """Raises H3Error when a kernel enqueued earlier on `device` has recorded a failure
    (a bounded wait that gave up, an out-of-range label).  The word is read without a
    device synchronisation, so a failure shows up at the first check after the kernel
    that recorded it has run; h3_device_error clears it."""
    code = device_error_peek(device)
    if code:
        msg = load().h3_status_string(code).decode()
        raise H3Error(f"{where}: an earlier kernel on cuda:{device} reported: {msg} "
                      f"(status {code}); read and clear it with h3_device_error")
