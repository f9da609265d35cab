"""The decoder-layer op mix built from this library's ops (Llama-7B shaped by default).

Per layer, on x [B, T, d_model]:
    qkv = FusedRMSNormLinear(d_model, 3 * d_model)(x)          RMSNorm fused into the QKV GEMM
    o   = flash_attn_forward(q, k, v, causal=True)               q, k, v are strided views of qkv;
                                                                  o is written in [B, T, H, D]
    y   = Int8Linear(d_model, d_model)(o)                        O projection (quantise + int8 GEMM)
    u   = Int8Linear(d_model, d_ff)(y)                           MLP up projection
The O projection's GEMM also quantises its own output for the MLP-up projection
(``int8_gemm_dequant_requant``): y goes from the tensor-memory accumulator to int8 codes and
row scales without an fp16 round trip through HBM and without a separate quantise pass; the
codes are bit-identical to ``quantize_symmetric(y)``.
This is the composition the reference's notebook builds from its modules
(notebooks/dev_walkthrough.ipynb, CustomTransformerBlock) reduced to the ops of the
benchmark's decoder-layer workload; there is no residual, activation or down projection.
Activations never take an extra copy between ops: attention reads q/k/v out of the QKV
output through strides and writes its output in the layout the O projection reads.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .flash_attn import flash_attn_forward
from .int8_gemm import int8_gemm_dequant_nk, int8_gemm_dequant_requant, quantize_symmetric

__all__ = ["DecoderLayerOps"]


class DecoderLayerOps(nn.Module):
    def __init__(self, d_model: int = 4096, n_heads: int = 32, d_ff: int = 11008,
                 dtype: torch.dtype = torch.bfloat16, init_std: float = 0.02):
        super().__init__()
        from . import FusedRMSNormLinear, Int8Linear

        assert d_model % n_heads == 0
        self.d_model, self.n_heads, self.d_ff = d_model, n_heads, d_ff
        self.head_dim = d_model // n_heads
        self.qkv = FusedRMSNormLinear(d_model, 3 * d_model).to(dtype)
        self.o_proj = Int8Linear(d_model, d_model)
        self.up = Int8Linear(d_model, d_ff)
        self.init_std = init_std
        self.dtype = dtype

    @torch.no_grad()
    def init_weights(self, generator: torch.Generator | None = None) -> None:
        """Random init w ~ N(0, init_std) for the three projections (on the module's device),
        and quantisation of the two int8 weights."""
        dev = self.qkv.w_lin.device
        std = self.init_std
        self.qkv.w_lin.copy_((torch.randn(self.qkv.w_lin.shape, generator=generator) * std).to(self.dtype))
        w_o = (torch.randn(self.d_model, self.d_model, generator=generator) * std).to(self.dtype).to(dev)
        w_u = (torch.randn(self.d_ff, self.d_model, generator=generator) * std).to(self.dtype).to(dev)
        self.o_proj.quantize_weights(w_o)
        self.up.quantize_weights(w_u)

    def forward(self, x: torch.Tensor, return_intermediates: bool = False):
        B, T, d = x.shape
        H, Dh = self.n_heads, self.head_dim
        qkv = self.qkv(x.reshape(B * T, d)).view(B, T, 3, H, Dh)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # [B, H, T, Dh] views
        attn = torch.empty(B, T, H, Dh, dtype=x.dtype, device=x.device)
        flash_attn_forward(q, k, v, causal=True, out=attn.transpose(1, 2))
        a_q, a_s = quantize_symmetric(attn.view(B * T, d))
        res = int8_gemm_dequant_requant(a_q, self.o_proj.w_q, a_s, self.o_proj.scale_w, "nk",
                                        return_output=return_intermediates)
        y_q, y_s = res[0], res[1]
        u = int8_gemm_dequant_nk(y_q, self.up.w_q, y_s, self.up.scale_w)
        if return_intermediates:
            return u.view(B, T, self.d_ff), {"qkv": qkv, "attn": attn, "y": res[2], "y_q": y_q, "y_s": y_s}
        return u.view(B, T, self.d_ff)

    def flops(self, B: int, T: int) -> dict:
        """Algorithmic work of one layer: GEMM ops 2*M*N*K, causal attention half of dense."""
        M, d = B * T, self.d_model
        return {
            "qkv": 2.0 * M * d * 3 * d,
            "attention": 4.0 * B * self.n_heads * T * T * self.head_dim / 2,
            "o_proj": 2.0 * M * d * d,
            "mlp_up": 2.0 * M * d * self.d_ff,
        }
