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
def attention_fp32(q, k, v, causal: bool, scale: float | None = None, row_block: int | None = None) -> torch.Tensor:
    """q [B,H,M,D], k/v [B,H,N,D] (any dtype/device) -> fp32 CPU [B,H,M,D].

    ``row_block`` evaluates the query rows in blocks of that many rows (the same arithmetic
    per row), so long sequences need only a [row_block, N] score matrix at a time."""
    qf = q.detach().to("cpu", torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    D = qf.shape[-1]
    sc = D ** -0.5 if scale is None else scale
    M, N = qf.shape[-2], kf.shape[-2]
    step = M if row_block is None else max(1, int(row_block))
    outs = []
    for r0 in range(0, M, step):
        r1 = min(M, r0 + step)
        s = torch.matmul(qf[..., r0:r1, :], kf.transpose(-1, -2)) * sc
        if causal:
            mask = torch.arange(N)[None, :] > torch.arange(r0, r1)[:, None]
            s = s.masked_fill(mask, float("-inf"))
        p = torch.softmax(s, dim=-1)
        outs.append(torch.matmul(p, vf))
    return outs[0] if len(outs) == 1 else torch.cat(outs, dim=-2)


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


@torch.no_grad()
def attention_lse_fp32(q, k, v, causal: bool, scale: float | None = None) -> torch.Tensor:
    """Per query row, ln(sum over visible keys of exp(scale * q.k)) in fp32 on the CPU:
    [B,H,M].  The quantity the reference's forward-with-LSE stores,
    L_i = m_i + log(l_i) (kernels/flash_attn/flash_attn_bwd.py:118-119)."""
    qf = q.detach().to("cpu", torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    D = qf.shape[-1]
    sc = D ** -0.5 if scale is None else scale
    s = torch.matmul(qf, kf.transpose(-1, -2)) * sc
    if causal:
        M, N = s.shape[-2], s.shape[-1]
        s = s.masked_fill(torch.arange(N)[None, :] > torch.arange(M)[:, None], float("-inf"))
    return torch.logsumexp(s, dim=-1)


def attention_grad_fp32(q, k, v, dout, causal: bool, scale: float | None = None):
    """(dq, dk, dv) of sum(O * dout) for O = attention_fp32(q, k, v, causal, scale), by fp32
    autograd on the CPU.  These are the gradients the reference's backward describes
    (kernels/flash_attn/flash_attn_bwd.py:13-19: dV = P^T dO, dP = dO V^T,
    dS = P (dP - Delta), dQ = scale dS K, dK = scale dS^T Q).  K/V with fewer heads than Q are
    repeat_interleave'd first, so their gradients sum over the query heads that share them."""
    qf = q.detach().to("cpu", torch.float32).requires_grad_(True)
    kf = k.detach().to("cpu", torch.float32).requires_grad_(True)
    vf = v.detach().to("cpu", torch.float32).requires_grad_(True)
    rep = qf.shape[1] // kf.shape[1]
    kk = kf.repeat_interleave(rep, dim=1) if rep > 1 else kf
    vv = vf.repeat_interleave(rep, dim=1) if rep > 1 else vf
    D = qf.shape[-1]
    sc = D ** -0.5 if scale is None else scale
    with torch.enable_grad():
        s = torch.matmul(qf, kk.transpose(-1, -2)) * sc
        if causal:
            M, N = s.shape[-2], s.shape[-1]
            s = s.masked_fill(torch.arange(N)[None, :] > torch.arange(M)[:, None], float("-inf"))
        o = torch.matmul(torch.softmax(s, dim=-1), vv)
        o.backward(dout.detach().to("cpu", torch.float32))
    return qf.grad, kf.grad, vf.grad
