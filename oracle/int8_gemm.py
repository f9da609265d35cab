"""int8 GEMM + dequant — restatement (test infrastructure).

int32 accumulator: kernels/int8_gemm/int8_gemm.py:59-78 (exact int32 sum over K), computed
by the C restatement in ``int8_gemm_ref.c`` (OpenMP) with a numpy fallback.
Dequant epilogue: kernels/int8_gemm/int8_gemm.py:81-89:
    out = acc.to(float32) * sa[:, None] * sb[None, :]   (left to right, fp32 RN)  (:84)
    C = out.to(float16)                                 (RN)                      (:88)
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compiles int8_gemm_ref.c into oracle/_build/liboracle.so (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _load():
    global _lib
    if _lib is None and os.path.exists(_SO):
        lib = ctypes.CDLL(_SO)
        for name in ("oracle_int8_gemm_i32_nk", "oracle_int8_gemm_i32_kn"):
            f = getattr(lib, name)
            f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                          ctypes.c_int64, ctypes.c_int]
        _lib = lib
    return _lib


def _np(x, dtype):
    try:
        import torch

        if isinstance(x, torch.Tensor):
            x = x.detach().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(x, dtype=dtype))


def int8_gemm_i32(A, B, b_layout: str = "kn", threads: int | None = None) -> np.ndarray:
    """Exact int32 ``A @ B`` with A int8 [M,K] and B int8 [K,N] ("kn") or [N,K] ("nk")."""
    a = _np(A, np.int8)
    b = _np(B, np.int8)
    M, K = a.shape
    N = b.shape[1] if b_layout == "kn" else b.shape[0]
    c = np.empty((M, N), dtype=np.int32)
    lib = _load()
    nt = threads or os.cpu_count() or 1
    if lib is not None:
        fn = lib.oracle_int8_gemm_i32_kn if b_layout == "kn" else lib.oracle_int8_gemm_i32_nk
        fn(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K, nt)
        return c
    bk = b if b_layout == "kn" else b.T
    return (a.astype(np.int64) @ bk.astype(np.int64)).astype(np.int32)


def dequant_f16(acc: np.ndarray, sa, sb) -> np.ndarray:
    """fp16((fp32(acc) * sa[m]) * sb[n]) with round-to-nearest at every step."""
    sa = _np(sa, np.float32)
    sb = _np(sb, np.float32)
    out = acc.astype(np.float32) * sa[:, None]
    out = out * sb[None, :]
    return out.astype(np.float16)


def int8_gemm_dequant(A, B, sa, sb, b_layout: str = "kn", threads: int | None = None) -> np.ndarray:
    return dequant_f16(int8_gemm_i32(A, B, b_layout, threads), sa, sb)
