"""Flash attention with gradients on sm_100a: a forward that also returns the log-sum-exp, and
the backward (tcgen05 + TMEM + TMA kernels reached through the C ABI).

Drop-in for the reference's ``kernels/flash_attn/flash_attn_bwd.py``: ``FlashAttnFunction``
(:245-334, a ``torch.autograd.Function`` with ``forward(ctx, q, k, v, causal=True, block_m=64,
block_n=64)``) and ``flash_attn_with_grad(q, k, v, causal=True, block_m=64, block_n=64)``
(:337-343).  The reference's kernels cannot run as written (the head dimension ``D`` they use
at :85 and :190 is never defined), so the contract here is the one they describe: the forward
stores ``L = m + log(l)`` per query row (:118-119), the backward recomputes
``P = exp(scale * Q K^T - L)`` and forms ``dV = P^T dO``, ``dS = P * (dO V^T - Delta)`` with
``Delta = rowsum(dO * O)`` (:293), ``dQ = scale * dS K`` and ``dK = scale * dS^T Q``.
Unlike the reference (atomic dQ, :217-220) every gradient is summed in a fixed order.

Superset, as in the forward: bf16 as well as fp16, any M and N, an optional softmax scale,
head dims other than 64 / 128 (zero-padded), and K / V with fewer heads than Q (the gradients
of a shared K / V head are the sums over its query heads, accumulated inside the kernel).
"""

from __future__ import annotations

import torch

from . import _lib
from ._common import dtype_code, ptr, require, require_cuda, stream_for

__all__ = ["flash_attn_forward_lse", "FlashAttnFunction", "flash_attn_with_grad"]

_TILE = 128


def _lse_ld(M: int) -> int:
    return max(_TILE, -(-M // _TILE) * _TILE)


def _vec_ok(t: torch.Tensor) -> bool:
    """A [B, H, S, D] tensor the kernels can read / write with 16-byte vectors and TMA."""
    return t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:3]) and t.data_ptr() % 16 == 0


def _prep(t: torch.Tensor) -> torch.Tensor:
    return t if _vec_ok(t) else t.contiguous()


def _check(q, k, v):
    require(isinstance(q, torch.Tensor) and isinstance(k, torch.Tensor) and isinstance(v, torch.Tensor),
            "q, k, v must be tensors")
    require(q.dtype in (torch.float16, torch.bfloat16) and q.is_cuda, "q must be a CUDA fp16/bf16 tensor")
    require(k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share a dtype")
    require_cuda("flash_attn_with_grad", q, k, v)
    require(q.dim() == 4 and k.dim() == 4 and v.dim() == 4, "q, k, v must be [B, H, seq, D]")
    B, H, M, D = q.shape
    N = k.shape[2]
    H_kv = k.shape[1]
    require(H_kv > 0 and H % H_kv == 0 and k.shape == (B, H_kv, N, D) and v.shape == (B, H_kv, N, D),
            "k and v must be [B, H_kv, N, D] matching q, with H_kv dividing H")
    require(0 < D <= 128, f"head dim {D} not supported (1..128)")
    require(N > 0, "need at least one key")
    return B, H, H_kv, M, N, D


def _padded(t: torch.Tensor, Dp: int) -> torch.Tensor:
    return t if t.shape[-1] == Dp else torch.nn.functional.pad(t, (0, Dp - t.shape[-1]))


def _forward_lse(q, k, v, causal: bool, scale: float):
    """(out, lse_buf) for D in {64, 128}; lse_buf is [B*H, lse_ld] fp32."""
    B, H, M, D = q.shape
    H_kv, N = k.shape[1], k.shape[2]
    q, k, v = _prep(q), _prep(k), _prep(v)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    ld = _lse_ld(M)
    lse = torch.empty((B * H, ld), dtype=torch.float32, device=q.device)
    if out.numel():
        _lib.call(
            "lk_flash_attn_fwd_lse", ptr(q), ptr(k), ptr(v), ptr(out), ptr(lse), ld, dtype_code(q.dtype),
            B, H, H_kv, M, N, D,
            _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), _lib.i64_array(v.stride()),
            _lib.i64_array(out.stride()), 1 if causal else 0, scale, stream_for(q.device),
        )
    return out, lse


def flash_attn_forward_lse(q, k, v, causal=True, softmax_scale=None):
    """``(out, lse)``: the attention output and, per query row, ``lse = ln sum_n exp(scale q.k_n)``
    over the visible keys (``[B, H, M]`` fp32), as the reference's forward with LSE stores it
    (flash_attn_bwd.py:118-119)."""
    B, H, H_kv, M, N, D = _check(q, k, v)
    scale = float(softmax_scale) if softmax_scale is not None else float(D) ** -0.5
    Dp = 64 if D <= 64 else 128
    out, lse = _forward_lse(_padded(q, Dp), _padded(k, Dp), _padded(v, Dp), causal, scale)
    return out[..., :D], lse[:, :M].view(B, H, M)


def _backward(q, k, v, out, dout, lse, causal: bool, scale: float):
    """dq, dk, dv for D in {64, 128}; k / v may have fewer heads than q."""
    B, H, M, D = q.shape
    H_kv, N = k.shape[1], k.shape[2]
    q, k, v, out, dout = (_prep(t) for t in (q, k, v, out, dout))
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    delta = torch.empty_like(lse)
    strides = [s for t in (q, k, v, out, dout, dq, dk, dv) for s in t.stride()]
    _lib.call(
        "lk_flash_attn_bwd", ptr(q), ptr(k), ptr(v), ptr(out), ptr(dout), ptr(lse), lse.shape[1],
        ptr(dq), ptr(dk), ptr(dv), ptr(delta), dtype_code(q.dtype), B, H, H_kv, M, N, D,
        _lib.i64_array(strides), 1 if causal else 0, scale, stream_for(q.device),
    )
    return dq, dk, dv


class FlashAttnFunction(torch.autograd.Function):
    """Flash attention forward + backward (flash_attn_bwd.py:245-334).

    ``FlashAttnFunction.apply(q, k, v, causal=True, block_m=64, block_n=64, softmax_scale=None)``;
    q [B, H, M, D], k / v [B, H_kv, N, D], fp16 / bf16 CUDA.  The tile arguments are accepted
    and validated for signature compatibility; the sm_100a kernels use their own 128-row tiles
    and any M, N."""

    @staticmethod
    def forward(ctx, q, k, v, causal=True, block_m=64, block_n=64, softmax_scale=None):
        for name, val in (("block_m", block_m), ("block_n", block_n)):
            require(isinstance(val, int) and val > 0, f"{name} must be a positive int")
        B, H, H_kv, M, N, D = _check(q, k, v)
        scale = float(softmax_scale) if softmax_scale is not None else float(D) ** -0.5
        Dp = 64 if D <= 64 else 128
        qp, kp, vp = _padded(q, Dp), _padded(k, Dp), _padded(v, Dp)
        out, lse = _forward_lse(qp, kp, vp, causal, scale)
        ctx.save_for_backward(qp, kp, vp, out, lse)
        ctx.causal, ctx.scale, ctx.D = bool(causal), scale, D
        return out[..., :D] if Dp != D else out

    @staticmethod
    def backward(ctx, dout):
        qp, kp, vp, out, lse = ctx.saved_tensors
        D = ctx.D
        Dp = qp.shape[-1]
        dq, dk, dv = _backward(qp, kp, vp, out, _padded(dout.to(qp.dtype), Dp), lse, ctx.causal, ctx.scale)
        if Dp != D:
            dq, dk, dv = dq[..., :D], dk[..., :D], dv[..., :D]
        return dq, dk, dv, None, None, None, None


def flash_attn_with_grad(q, k, v, causal=True, block_m=64, block_n=64, softmax_scale=None):
    """Flash attention whose output supports ``.backward()`` / ``torch.autograd.grad``
    (flash_attn_bwd.py:337-343)."""
    return FlashAttnFunction.apply(q, k, v, causal, block_m, block_n, softmax_scale)
