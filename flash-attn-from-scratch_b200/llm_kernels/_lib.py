"""ctypes binding of the C ABI in ``include/llm_kernels_b200.h`` (``liblk_b200.so``).

This is the only way the Python layer reaches the GPU: every op calls one of these entry
points with raw device pointers, element strides and torch's current CUDA stream.  There is
no other code path — if the library is missing, the ops raise instead of computing anything.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblk_b200.so")

# Status codes (lk_status) and dtype codes (lk_dtype) of the header.
LK_OK = 0
LK_ERR_INVALID_ARG = 1
LK_ERR_UNSUPPORTED = 2
LK_ERR_CUDA = 3
LK_ERR_TIMEOUT = 4
LK_ERR_ALIGNMENT = 5
LK_ERR_SCRATCH_LIMIT = 6
LK_PEER_HANDLE_BYTES = 64  # include/llm_kernels_b200.h

LK_F32, LK_F16, LK_BF16, LK_I8, LK_I32 = 0, 1, 2, 3, 4

# Failure-path test hooks (lk_inject).
LK_INJECT_NONE, LK_INJECT_FA_DROP_LOAD, LK_INJECT_GEMM_DROP_LOAD, LK_INJECT_SPLIT_SKIP_PUBLISH = 0, 1, 2, 3
LK_INJECT_REQUANT_SKIP_PUBLISH = 4

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_pi64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/llm_kernels_b200.h one for one.
SIGNATURES = {
    "lk_status_string": (ctypes.c_char_p, [_i]),
    "lk_last_cuda_error": (_i, []),
    "lk_version": (_i, []),
    "lk_set_device": (_i, [_i]),
    "lk_device_status": (_i, [ctypes.POINTER(ctypes.c_int)]),
    "lk_clear_device_status": (_i, []),
    "lk_debug_set_wait_limit": (_i, [_i64]),
    "lk_debug_inject": (_i, [_i, _i, _i]),
    "lk_quantize_symmetric": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "lk_int8_gemm_dequant": (_i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "lk_int8_gemm_i32": (_i, [_p, _i64, _p, _i64, _i, _p, _i64, _i64, _i64, _i64, _p]),
    "lk_int8_gemm_requant_workspace_bytes": (_i64, [_i64]),
    "lk_int8_gemm_dequant_requant": (
        _i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _p],
    ),
    "lk_int8_gemm_dequant_scatter": (
        _i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _i64, _p],
    ),
    "lk_int8_gemm_dequant_multicast": (
        _i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    ),
    "lk_peer_export": (_i, [_i, _p, _p, _pi64]),
    "lk_peer_open": (_i, [_i, _p, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "lk_peer_close": (_i, [_i, _p, _i64]),
    "lk_flash_attn_fwd": (
        _i,
        [_p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64, _pi64, _i, _f, _p],
    ),
    "lk_flash_attn_fwd_gqa": (
        _i,
        [_p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64, _pi64, _i, _f, _p],
    ),
    "lk_flash_attn_fwd_lse": (
        _i,
        [_p, _p, _p, _p, _p, _i64, _i, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64, _pi64, _i, _f, _p],
    ),
    "lk_flash_attn_bwd": (
        _i,
        [_p, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _i, _f, _p],
    ),
    "lk_rmsnorm_linear_fold": (_i, [_p, _i, _p, _p, _i, _i64, _i64, _p]),
    "lk_rmsnorm_linear": (_i, [_p, _i64, _p, _p, _i64, _i, _i64, _i64, _i64, _f, _p, _p]),
    "lk_fused_rmsnorm_linear": (_i, [_p, _p, _p, _p, _f, _i64, _i64, _i64, _i, _p, _p, _p]),
    "lk_rmsnorm_linear_noalloc": (_i, [_p, _i64, _p, _p, _i64, _i, _i64, _i64, _i64, _f, _p]),
}

_lib = None
_lock = threading.Lock()


class LKError(RuntimeError):
    """A C-ABI call returned a failure status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        msg = f"{fn}: {status_string(status)} (status {status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


def load() -> ctypes.CDLL:
    """Loads ``liblk_b200.so`` (once) and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"llm_kernels: native library {LIB_PATH} is missing; build it with "
                "`python flash-attn-from-scratch_b200/build.py` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    try:
        return load().lk_status_string(int(status)).decode()
    except Exception:  # pragma: no cover - only when the library itself failed to load
        return "unknown"


def call(name: str, *args) -> None:
    """Calls entry point ``name`` and raises LKError on a non-zero status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != LK_OK:
        detail = ""
        if st == LK_ERR_CUDA:
            detail = f"cudaError {lib.lk_last_cuda_error()}"
        raise LKError(name, st, detail)


def i64_array(vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


_tls = threading.local()


def set_device(index: int) -> None:
    """Makes device ``index`` current for the library on this thread (cached)."""
    if getattr(_tls, "device", None) != index:
        call("lk_set_device", int(index))
        _tls.device = index


def device_status() -> tuple[int, int, int, int]:
    """Synchronises and returns the device status word (code, site, block, thread)."""
    out = (ctypes.c_int * 4)()
    st = load().lk_device_status(out)
    if st not in (LK_OK, LK_ERR_TIMEOUT):
        raise LKError("lk_device_status", st)
    return tuple(out)


def clear_device_status() -> None:
    call("lk_clear_device_status")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
