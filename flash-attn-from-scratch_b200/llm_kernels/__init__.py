"""
llm_kernels (B200 / sm_100a)
============================
Drop-in replacement for the reference ``llm_kernels`` package (llm_kernels/__init__.py:1-135):
the same four functions and three ``nn.Module`` wrappers, backed by hand-written sm_100a
kernels reached through the C ABI in ``include/llm_kernels_b200.h``.

>>> import llm_kernels
>>> out = llm_kernels.flash_attn_forward(q, k, v, causal=True)
>>> out = llm_kernels.int8_gemm_dequant_fwd(A_q, B_q, sa, sb)
>>> out = llm_kernels.fused_rmsnorm_linear(x, w_norm, w_lin)
>>> out = llm_kernels.flash_attn_with_grad(q, k, v, causal=True); out.sum().backward()

There is no CPU or PyTorch fallback: every op runs its CUDA kernel or raises.
"""

import torch
import torch.nn as nn

from ._common import LKInputError
from ._lib import LKError, device_status, clear_device_status
from .flash_attn import flash_attn_forward
from .flash_attn_bwd import FlashAttnFunction, flash_attn_forward_lse, flash_attn_with_grad
from .fused_rmsnorm_linear import fused_rmsnorm_linear, fold_norm_weight, clear_fold_cache
from .int8_gemm import (
    int8_gemm_dequant_fwd,
    int8_gemm_dequant_auto,
    int8_gemm_dequant_nk,
    int8_gemm_dequant_requant,
    int8_gemm_i32,
    quantize_symmetric,
)


class FlashAttention(nn.Module):
    """Drop-in for scaled_dot_product_attention (llm_kernels/__init__.py:30-52).

    >>> attn = FlashAttention(causal=True)
    >>> out = attn(q, k, v)   # [B, H, M, D] fp16 / bf16
    """

    def __init__(self, causal: bool = True, block_m: int = 64, block_n: int = 64):
        super().__init__()
        self.causal = causal
        self.block_m = block_m
        self.block_n = block_n

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        return flash_attn_forward(q, k, v, causal=self.causal, block_m=self.block_m, block_n=self.block_n)

    def extra_repr(self) -> str:
        return f"causal={self.causal}, block_m={self.block_m}, block_n={self.block_n}"


class FusedRMSNormLinear(nn.Module):
    """Fused RMSNorm + Linear layer (llm_kernels/__init__.py:55-79).

    Equivalent to ``nn.Linear(d_in, d_out, bias=False)(nn.RMSNorm(d_in)(x))``.  Parameters
    ``w_norm`` [d_in] and ``w_lin`` [d_out, d_in] keep the reference's names, shapes and fp16
    default dtype, so its state_dicts load unchanged.

    >>> layer = FusedRMSNormLinear(d_in=4096, d_out=4096)
    >>> y = layer(x)   # [B, D_out]
    """

    def __init__(self, d_in: int, d_out: int, eps: float = 1e-6):
        super().__init__()
        self.d_in = d_in
        self.d_out = d_out
        self.eps = eps
        self.w_norm = nn.Parameter(torch.ones(d_in, dtype=torch.float16))
        self.w_lin = nn.Parameter(torch.empty(d_out, d_in, dtype=torch.float16))
        nn.init.kaiming_uniform_(self.w_lin, a=5**0.5)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_rmsnorm_linear(x, self.w_norm, self.w_lin, self.eps)

    def extra_repr(self) -> str:
        return f"d_in={self.d_in}, d_out={self.d_out}, eps={self.eps}"


class Int8Linear(nn.Module):
    """int8 linear layer with fused dequantisation (llm_kernels/__init__.py:82-121).

    Buffers ``w_q`` [d_out, d_in] int8 and ``scale_w`` [d_out] fp32 as in the reference.  The
    forward quantises x per row and runs the int8 GEMM with the weight in its stored [N, K]
    layout — the reference transposed it into a fresh [K, N] copy on every call
    (llm_kernels/__init__.py:115); the integer result is the same.

    >>> layer = Int8Linear(d_in=4096, d_out=4096)
    >>> layer.quantize_weights(w_fp16)
    >>> y = layer(x)   # [B, D_out] fp16
    """

    def __init__(self, d_in: int, d_out: int):
        super().__init__()
        self.d_in = d_in
        self.d_out = d_out
        self.register_buffer("w_q", torch.zeros(d_out, d_in, dtype=torch.int8))
        self.register_buffer("scale_w", torch.ones(d_out, dtype=torch.float32))

    @torch.no_grad()
    def quantize_weights(self, w: torch.Tensor):
        """Quantise an fp16/bf16/fp32 weight [D_out, D_in] and store it as int8."""
        self.w_q, self.scale_w = quantize_symmetric(w)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x : [..., D_in] fp16 / bf16 / fp32 -> [..., D_out] fp16."""
        lead = x.shape[:-1]
        x_q, scale_x = quantize_symmetric(x.reshape(-1, x.shape[-1]))
        y = int8_gemm_dequant_nk(x_q, self.w_q.contiguous(), scale_x, self.scale_w)
        return y.reshape(*lead, self.d_out)

    def extra_repr(self) -> str:
        return f"d_in={self.d_in}, d_out={self.d_out}"


from .decoder import DecoderLayerOps  # noqa: E402  (uses the modules above)

__all__ = [
    # functions
    "flash_attn_forward",
    "int8_gemm_dequant_fwd",
    "quantize_symmetric",
    "fused_rmsnorm_linear",
    # modules
    "FlashAttention",
    "FusedRMSNormLinear",
    "Int8Linear",
    # training path (the reference's kernels/flash_attn/flash_attn_bwd.py)
    "FlashAttnFunction",
    "flash_attn_with_grad",
    "flash_attn_forward_lse",
]
