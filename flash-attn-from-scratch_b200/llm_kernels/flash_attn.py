"""Flash-attention forward on sm_100a (tcgen05 + TMEM + TMA).

Drop-in for the reference's ``kernels/flash_attn/flash_attn_fwd.py:131-156``
(``flash_attn_forward``), which dispatched to a non-causal (:6-64) or causal (:67-128) Triton
kernel.  Same arguments and defaults; as a superset it also accepts bf16, ragged M/N (no
tile-multiple requirement), an optional ``softmax_scale``, and K/V with fewer heads than Q
(grouped-query / multi-query attention, the reference's ``experiments/attention_ablation.py``
GroupedQueryAttention and MultiQueryAttention) read in place without repeating them.
"""

from __future__ import annotations

import torch

from . import _lib
from ._common import dtype_code, ptr, require, require_cuda, stream_for

__all__ = ["flash_attn_forward"]


def flash_attn_forward(q, k, v, causal=True, block_m=64, block_n=64, softmax_scale=None, out=None):
    """``O = softmax(Q K^T * scale [+ causal mask]) V`` for ``[B, H, M, D]`` tensors.

    Args:
        q : [B, H, M, D] fp16 / bf16, CUDA (any strides with a contiguous last dim)
        k, v : [B, H_kv, N, D], same dtype and device; H_kv divides H and query head h
            attends to K/V head h // (H // H_kv) (``repeat_interleave`` order,
            attention_ablation.py:125-127).  H_kv = H is ordinary attention; a single K/V
            head ``expand``-ed to H heads (attention_ablation.py:87-88) is read in place.
        causal : mask keys n > m (top-left aligned, flash_attn_fwd.py:118)
        block_m, block_n : accepted for signature compatibility; the sm_100a kernel uses
            its own 128-row tiles and handles any M, N.
        softmax_scale : defaults to D**-0.5 (flash_attn_fwd.py:50)
        out : optional preallocated ``[B, H, M, D]`` output (any strides with a contiguous
            last dim), e.g. a ``[B, M, H, D]`` buffer viewed with ``transpose(1, 2)`` so the
            next projection reads it without a copy.

    Returns:
        out : like ``q`` (``torch.empty_like(q)``, flash_attn_fwd.py:136), or ``out``
    """
    require(isinstance(q, torch.Tensor) and isinstance(k, torch.Tensor) and isinstance(v, torch.Tensor), "q, k, v must be tensors")
    require(q.dtype in (torch.float16, torch.bfloat16) and q.is_cuda, "q must be a CUDA fp16/bf16 tensor")
    require(k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share a dtype")
    dev = require_cuda("flash_attn_forward", q, k, v)
    require(q.dim() == 4 and k.dim() == 4 and v.dim() == 4, "q, k, v must be [B, H, seq, D]")
    for name, val in (("block_m", block_m), ("block_n", block_n)):
        require(isinstance(val, int) and val > 0, f"{name} must be a positive int")
    B, H, M, D = q.shape
    N = k.shape[2]
    if H > 1 and k.shape == (B, H, N, D) and v.shape == k.shape and k.stride(1) == 0 and v.stride(1) == 0:
        k, v = k[:, :1], v[:, :1]  # one K/V head broadcast over the query heads
    H_kv = k.shape[1]
    require(H_kv > 0 and H % H_kv == 0 and k.shape == (B, H_kv, N, D) and v.shape == (B, H_kv, N, D),
            "k and v must be [B, H_kv, N, D] matching q, with H_kv dividing H")
    require(0 < D <= 128, f"head dim {D} not supported (1..128)")
    scale = float(softmax_scale) if softmax_scale is not None else float(D) ** -0.5
    if out is not None:
        require(isinstance(out, torch.Tensor) and out.shape == q.shape and out.dtype == q.dtype
                and out.device == q.device, "out must match q's shape, dtype and device")
    if D not in (64, 128):
        # The tcgen05 kernels are built for D = 64 and 128; other head dims are zero-padded
        # (zero columns add nothing to Q K^T, and the padded output columns are dropped).
        Dp = 64 if D < 64 else 128
        pad = lambda t: torch.nn.functional.pad(t, (0, Dp - D))
        padded = flash_attn_forward(pad(q), pad(k), pad(v), causal, block_m, block_n, softmax_scale=scale)
        res = out if out is not None else torch.empty_like(q)
        res.copy_(padded[..., :D])
        return res
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    if out is not None and out.stride(-1) == 1 and all(s % 8 == 0 for s in out.stride()[:3]) \
            and out.data_ptr() % 16 == 0:
        pass
    elif out is not None:
        res = flash_attn_forward(q, k, v, causal, block_m, block_n, softmax_scale=scale)
        out.copy_(res)
        return out
    else:
        out = torch.empty_like(q)
        if out.stride(-1) != 1:
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if out.numel() == 0:
        return out
    require(N > 0, "flash_attn_forward: need at least one key")
    s = stream_for(dev)
    heads = (H,) if H_kv == H else (H, H_kv)
    _lib.call(
        "lk_flash_attn_fwd" if H_kv == H else "lk_flash_attn_fwd_gqa",
        ptr(q), ptr(k), ptr(v), ptr(out), dtype_code(q.dtype),
        B, *heads, M, N, D,
        _lib.i64_array(q.stride()), _lib.i64_array(k.stride()),
        _lib.i64_array(v.stride()), _lib.i64_array(out.stride()),
        1 if causal else 0, scale, s,
    )
    return out
