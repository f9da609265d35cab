"""Shared host-side helpers: argument checks, dtype codes, stream/device binding."""

from __future__ import annotations

import torch

from . import _lib


class LKInputError(AssertionError, ValueError):
    """Invalid arguments.

    The reference validated with bare ``assert`` (kernels/flash_attn/flash_attn_fwd.py:132-135,
    kernels/int8_gemm/int8_gemm.py:113-120), so callers may catch AssertionError; this class is
    also a ValueError so it survives ``python -O``-style expectations."""


def require(cond: bool, msg: str) -> None:
    if not cond:
        raise LKInputError(msg)


_DTYPE_CODE = {
    torch.float32: _lib.LK_F32,
    torch.float16: _lib.LK_F16,
    torch.bfloat16: _lib.LK_BF16,
    torch.int8: _lib.LK_I8,
    torch.int32: _lib.LK_I32,
}


def dtype_code(dt: torch.dtype) -> int:
    require(dt in _DTYPE_CODE, f"unsupported dtype {dt}")
    return _DTYPE_CODE[dt]


def require_cuda(name: str, *tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device; returns it.  There is no CPU path in this library."""
    dev = None
    for t in tensors:
        require(isinstance(t, torch.Tensor), f"{name}: expected tensors")
        require(t.is_cuda, f"{name}: inputs must be CUDA tensors (this library has no CPU path)")
        if dev is None:
            dev = t.device
        require(t.device == dev, f"{name}: all inputs must be on the same device")
    return dev


def stream_for(dev: torch.device) -> int:
    """Binds the library to ``dev`` and returns torch's current stream handle there."""
    _lib.set_device(dev.index if dev.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(dev).cuda_stream


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()
