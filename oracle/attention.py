"""Attention forward in fp32 on the CPU (test infrastructure).

The floating-point target: softmax(Q K^T * scale) V evaluated in fp32,
with the reference's causal convention — key n is visible to query m iff n <= m, top-left
aligned (kernels/flash_attn/flash_attn_fwd.py:118-119) — and its default scale D**-0.5
(flash_attn_fwd.py:50).  The reference tests compare against torch SDPA the same way
(tests/test_correctness.py:42, :57).
"""

from __future__ import annotations

import torch


@torch.no_grad()
def attention_fp32(q, k, v, causal: bool, scale: float | None = None) -> torch.Tensor:
    """q [B,H,M,D], k/v [B,H,N,D] (any dtype/device) -> fp32 CPU [B,H,M,D]."""
    qf = q.detach().to("cpu", torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    D = qf.shape[-1]
    sc = D ** -0.5 if scale is None else scale
    s = torch.matmul(qf, kf.transpose(-1, -2)) * sc
    if causal:
        M, N = s.shape[-2], s.shape[-1]
        mask = torch.arange(N)[None, :] > torch.arange(M)[:, None]
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf)


def attention_gqa_fp32(q, k, v, causal: bool, scale: float | None = None) -> torch.Tensor:
    """Grouped-query attention: q [B,H,M,D], k/v [B,H_kv,N,D] with H_kv dividing H.

    Restates the reference's GroupedQueryAttention (experiments/attention_ablation.py:118-141):
    K and V heads are repeat_interleave'd H // H_kv times along the head axis (:125-127), so
    query head h reads K/V head h // (H // H_kv); then the same softmax(Q K^T * scale) V.
    H_kv = 1 is MultiQueryAttention (:70-104)."""
    H, H_kv = q.shape[1], k.shape[1]
    assert H % H_kv == 0, "H_kv must divide H"
    rep = H // H_kv
    return attention_fp32(q, k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1), causal, scale)
