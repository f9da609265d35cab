"""Flash-attention training path on the GPU vs the oracle: the forward's log-sum-exp against
oracle.attention_lse_fp32 and dQ / dK / dV against oracle.attention_grad_fp32 (fp32 autograd of
softmax(Q K^T * scale) V on the CPU, from the same fp16 / bf16 inputs).

Tolerances.  LSE (fp32 output): max-abs 1e-3.  Gradients (fp16 / bf16 outputs):
  * relative error max |g - g_ref| / max(1, max |g_ref|) <= 1e-2 for every tensor and dtype
    (the relative-error definition of the RMSNorm+Linear tolerance, floored at 1 so tensors
    with small entries are held to 1e-2 absolute);
  * per element, |g - g_ref| / max(1, |g_ref|) <= 1e-2 in fp16 and <= 2e-2 in bf16: the MMAs
    take P and dS rounded to the input type, and bf16's 8-bit mantissa (relative step 2^-8)
    leaves about 1e-2 of error on sums with heavy cancellation.
The forward output keeps its own bound (test_flash_attn_gpu.py).
"""

import os

import numpy as np
import pytest
import torch

import llm_kernels
import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _scaled_err(got, ref):
    return ((got.float().cpu() - ref).abs() / ref.abs().clamp(min=1.0)).max().item()


def _rel_err(got, ref):
    return ((got.float().cpu() - ref).abs().max() / ref.abs().max().clamp(min=1.0)).item()


def _elem_tol(dtype):
    return 2e-2 if dtype == torch.bfloat16 else 1e-2


def _inputs(B, H, H_kv, M, N, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, M, D, generator=g).to(dtype)
    k = torch.randn(B, H_kv, N, D, generator=g).to(dtype)
    v = torch.randn(B, H_kv, N, D, generator=g).to(dtype)
    do = torch.randn(B, H, M, D, generator=g).to(dtype)
    return q, k, v, do


def _grads(q, k, v, do, causal, scale=None):
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = llm_kernels.flash_attn_with_grad(qd, kd, vd, causal, 64, 64, scale)
    out.backward(do.cuda())
    return out, qd.grad, kd.grad, vd.grad


def _check(q, k, v, do, causal, scale=None):
    out, dq, dk, dv = _grads(q, k, v, do, causal, scale)
    rdq, rdk, rdv = oracle.attention_grad_fp32(q, k, v, do, causal, scale)
    ref_out = oracle.attention_gqa_fp32(q, k, v, causal, scale)
    assert _scaled_err(out, ref_out) <= TOL
    for n, g, r in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert _rel_err(g, r) <= TOL, (n, _rel_err(g, r))
        assert _scaled_err(g, r) <= _elem_tol(q.dtype), (n, _scaled_err(g, r))
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
    assert dq.dtype == q.dtype and dk.dtype == k.dtype and dv.dtype == v.dtype


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("M,N", [(128, 128), (256, 256), (384, 384), (1024, 1024)])
def test_gradients_match_fp32_autograd(dtype, D, causal, M, N):
    _check(*_inputs(1, 2, 2, M, N, D, dtype, M + D), causal)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("M,N", [(1, 1), (5, 77), (200, 333), (333, 200), (129, 257), (700, 64), (64, 700)])
def test_gradients_ragged_and_rectangular(causal, M, N):
    """Tails of both the query and the key tiles; with causal and N > M the keys past the last
    query are seen by no query, and their dK, dV are exactly zero."""
    for dtype in (torch.bfloat16, torch.float16):
        q, k, v, do = _inputs(2, 3, 3, M, N, 128, dtype, M * 7 + N)
        _check(q, k, v, do, causal)
    if causal and N > M:
        _, _, dk, dv = _grads(q, k, v, do, True)
        assert bool((dk[:, :, M:] == 0).all()) and bool((dv[:, :, M:] == 0).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_forward_lse_matches_oracle(dtype, D, causal):
    q, k, v, _ = _inputs(2, 3, 3, 300, 333, D, dtype, 9 + D)
    out, lse = llm_kernels.flash_attn_forward_lse(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    assert lse.shape == (2, 3, 300) and lse.dtype == torch.float32
    assert (lse.cpu() - oracle.attention_lse_fp32(q, k, v, causal)).abs().max().item() <= 1e-3
    plain = llm_kernels.flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    assert torch.equal(out, plain)  # the LSE output does not change O


def test_golden_reference_backward_vectors():
    """The reference's own backward kernel, interpreted on the CPU (non-causal; its causal loop
    bounds are wrong, see tests/golden/make_golden.py), and its forward-with-LSE (both modes)."""
    g = np.load(os.path.join(GOLDEN, "flash_attn_bwd.npz"))
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    for causal in (0, 1):
        _, lse = llm_kernels.flash_attn_forward_lse(q.cuda(), k.cuda(), v.cuda(), causal=bool(causal))
        assert (lse.cpu() - torch.from_numpy(g[f"lse_causal{causal}"])).abs().max().item() <= 2e-3
    _, dq, dk, dv = _grads(q, k, v, do, False)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = torch.from_numpy(g[f"{name}_causal0"]).float()
        assert (got.float().cpu() - ref).abs().max().item() <= 1e-2, name


def test_grouped_query_odd_head_dim_scale_and_strided_views():
    # K/V shared by two query heads each; head dim 80 (zero-padded to 128); explicit scale
    q, k, v, do = _inputs(1, 4, 2, 200, 200, 80, torch.bfloat16, 21)
    _check(q, k, v, do, True, scale=0.2)
    # [B, T, H, D] storage on the GPU viewed as [B, H, T, D]: read through strides, no copy
    g = torch.Generator().manual_seed(22)
    x = torch.randn(2, 300, 4, 3, 64, generator=g).to(torch.float16).cuda()
    q, k, v = (x[:, :, :, i].transpose(1, 2) for i in range(3))
    assert q.stride(-1) == 1 and not q.is_contiguous()
    do = torch.randn(2, 4, 300, 64, generator=g).to(torch.float16)
    _check(q, k, v, do, True)


def test_backward_is_deterministic():
    """No atomics: two backward passes give identical bits."""
    q, k, v, do = _inputs(2, 4, 4, 1000, 1000, 128, torch.bfloat16, 23)
    a = _grads(q, k, v, do, True)
    b = _grads(q, k, v, do, True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_config2_shape_subset_of_heads():
    """Config-2 shape (B4 H32 N4096 D128 bf16, causal): the whole backward runs on the GPU;
    two (b, h) slices are checked against fp32 autograd on the CPU."""
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v, do = (torch.randn(4, 32, 4096, 128, generator=g, device="cuda").to(torch.bfloat16) for _ in range(4))
    _, dq, dk, dv = _grads(q, k, v, do, True)
    for b, h in ((0, 0), (3, 31)):
        sl = (slice(b, b + 1), slice(h, h + 1))
        rdq, rdk, rdv = oracle.attention_grad_fp32(q[sl], k[sl], v[sl], do[sl], True)
        for name, got, ref in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            assert _rel_err(got[sl], ref) <= TOL, (b, h, name)
            assert _scaled_err(got[sl], ref) <= _elem_tol(torch.bfloat16), (b, h, name)


def test_rejects_bad_inputs():
    q = torch.randn(1, 2, 64, 64, dtype=torch.float32, device="cuda")
    with pytest.raises(llm_kernels.LKInputError):
        llm_kernels.flash_attn_with_grad(q, q, q)
    q16 = q.half()
    with pytest.raises(llm_kernels.LKInputError):
        llm_kernels.flash_attn_with_grad(q16, q16[:, :, :, :32], q16)
