"""The oracle against golden vectors produced by the reference's own code (CPU only).

tests/golden/make_golden.py ran the reference here: quantize_symmetric and
_rmsnorm_linear_ref directly, the int8 GEMM and flash-attention Triton kernels under
TRITON_INTERPRET=1.  Passing these pins the oracle to the reference before it is used to
check the sm_100a kernels.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("case", ["f16", "f32", "bf16", "f16_wide", "f32_special"])
def test_quantize_bit_exact_vs_reference(case):
    g = _load("quantize")
    x = g[f"{case}_x"]
    x = _bf16(x) if case == "bf16" else torch.from_numpy(x)
    q, s = oracle.quantize_symmetric(x)
    np.testing.assert_array_equal(q, g[f"{case}_q"])
    ref_s = g[f"{case}_scale"]
    assert np.array_equal(np.isnan(s), np.isnan(ref_s))
    ok = ~np.isnan(ref_s)
    assert np.array_equal(s[ok].view(np.uint32), ref_s[ok].view(np.uint32))


@pytest.mark.parametrize("tag", ["sq", "rag"])
def test_int8_gemm_dequant_bit_exact_vs_reference_kernel(tag):
    g = _load("int8_gemm")
    C = oracle.int8_gemm_dequant(g[f"{tag}_A"], g[f"{tag}_B_kn"], g[f"{tag}_sa"], g[f"{tag}_sb"], "kn")
    np.testing.assert_array_equal(C.view(np.uint16), g[f"{tag}_C"].view(np.uint16))


@pytest.mark.parametrize("tag", ["sq", "rag"])
def test_int8_accumulator_layouts_agree(tag):
    g = _load("int8_gemm")
    A, B = g[f"{tag}_A"], g[f"{tag}_B_kn"]
    c_kn = oracle.int8_gemm_i32(A, B, "kn")
    c_nk = oracle.int8_gemm_i32(A, np.ascontiguousarray(B.T), "nk")
    c_np = (A.astype(np.int64) @ B.astype(np.int64))
    np.testing.assert_array_equal(c_kn, c_np)
    np.testing.assert_array_equal(c_nk, c_np)


@pytest.mark.parametrize("causal", [0, 1])
def test_attention_fp32_vs_reference_kernel(causal):
    g = _load("flash_attn")
    q, k, v = (torch.from_numpy(g[n]) for n in ("q", "k", "v"))
    ref = torch.from_numpy(g[f"out_causal{causal}"]).float()
    out = oracle.attention_fp32(q, k, v, causal=bool(causal))
    # the reference kernel stores fp16 and feeds PV with fp16 probabilities
    assert (out - ref).abs().max().item() < 1e-2


@pytest.mark.parametrize("tag", ["gqa", "mqa"])
@pytest.mark.parametrize("causal", [0, 1])
def test_attention_gqa_vs_reference_modules(tag, causal):
    """The grouped-query oracle against the reference's GroupedQueryAttention (2 K/V heads for
    8 query heads) and MultiQueryAttention modules run here in fp32."""
    g = _load("gqa")
    q, k, v = (torch.from_numpy(g[f"{tag}_{n}"]) for n in ("q", "k", "v"))
    assert k.shape[1] == (2 if tag == "gqa" else 1) and q.shape[1] == 8
    ref = torch.from_numpy(g[f"{tag}_out_causal{causal}"])
    out = oracle.attention_gqa_fp32(q, k, v, causal=bool(causal))
    assert (out - ref).abs().max().item() < 1e-5


def test_attention_gqa_head_mapping_is_repeat_interleave():
    """Query head h reads K/V head h // (H // H_kv), not h % H_kv: a planted modulo mapping
    must disagree with the golden outputs."""
    g = _load("gqa")
    q, k, v = (torch.from_numpy(g[f"gqa_{n}"]) for n in ("q", "k", "v"))
    ref = torch.from_numpy(g["gqa_out_causal0"])
    wrong = oracle.attention_fp32(q, k.repeat(1, 4, 1, 1), v.repeat(1, 4, 1, 1), causal=False)
    assert (wrong - ref).abs().max().item() > 1e-2


@pytest.mark.parametrize("tag", ["f32", "f16"])
def test_rmsnorm_linear_vs_reference(tag):
    g = _load("rmsnorm_linear")
    x, wn, wl = (torch.from_numpy(g[f"{tag}_{n}"]) for n in ("x", "w_norm", "w_lin"))
    y = oracle.rmsnorm_linear_ref(x, wn, wl, 1e-6, round_to_input_dtype=(tag == "f16"))
    ref = torch.from_numpy(g[f"{tag}_y"]).float()
    rel = (y - ref).abs().max() / ref.abs().max()
    assert rel.item() < (1e-6 if tag == "f32" else 2e-3)


def test_golden_vectors_reject_a_planted_rounding_mistake():
    """A quantiser that rounds half away from zero (a plausible bug) must fail the golden
    codes on the ties row, so the fixtures really discriminate the rounding mode."""
    g = _load("quantize")
    x = g["f32_special_x"].astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        scale = np.abs(x).max(-1) / np.float32(127)
        t = x / scale[:, None]
        wrong = np.where(np.isnan(t), 0, np.clip(np.sign(t) * np.floor(np.abs(t) + 0.5), -128, 127)).astype(np.int8)
    assert not np.array_equal(wrong[4], g["f32_special_q"][4])
    q, _ = oracle.quantize_symmetric(torch.from_numpy(x))
    np.testing.assert_array_equal(q, g["f32_special_q"])


@pytest.mark.parametrize("causal", [0, 1])
def test_attention_lse_vs_reference_forward_with_lse(causal):
    """The LSE the reference's forward-with-LSE kernel stores (flash_attn_bwd.py:118-119)."""
    g = _load("flash_attn_bwd")
    q, k, v = (torch.from_numpy(g[n]) for n in ("q", "k", "v"))
    lse = oracle.attention_lse_fp32(q, k, v, bool(causal))
    assert (lse - torch.from_numpy(g[f"lse_causal{causal}"])).abs().max().item() <= 2e-3
    out = oracle.attention_fp32(q, k, v, bool(causal))
    assert (out - torch.from_numpy(g[f"out_causal{causal}"]).float()).abs().max().item() <= 1e-2


def test_attention_grad_vs_reference_backward_kernel():
    """dQ, dK, dV of the reference's backward kernel (flash_attn_bwd.py:127-237, fp16 operands,
    fp16 atomics for dQ) on the non-causal case; the reference's causal loop bounds are wrong
    (make_golden.make_flash_attn_bwd), so only the non-causal gradients pin the oracle."""
    g = _load("flash_attn_bwd")
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    dq, dk, dv = oracle.attention_grad_fp32(q, k, v, do, False)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = torch.from_numpy(g[f"{name}_causal0"]).float()
        assert (got - ref).abs().max().item() <= 5e-3, name


def test_attention_grad_is_the_gradient_of_the_oracle_forward():
    """Finite differences of sum(O * dO) against the oracle's gradients (fp64 inputs), causal
    and not, with fewer K/V heads than Q heads: the gradients are those of attention_fp32 /
    attention_gqa_fp32."""
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 4, 9, 8, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 11, 8, generator=g, dtype=torch.float64)
    v = torch.randn(1, 2, 11, 8, generator=g, dtype=torch.float64)
    do = torch.randn(1, 4, 9, 8, generator=g, dtype=torch.float64)
    for causal in (False, True):
        dq, dk, dv = oracle.attention_grad_fp32(q, k, v, do, causal)
        f = lambda qq, kk, vv: (oracle.attention_gqa_fp32(qq, kk, vv, causal) * do.float()).sum().item()  # noqa: E731
        for t, grad, idx in ((q, dq, (0, 3, 8, 5)), (k, dk, (0, 1, 4, 2)), (v, dv, (0, 0, 10, 7))):
            e = 1e-2
            tp, tm = t.clone(), t.clone()
            tp[idx] += e
            tm[idx] -= e
            args_p = [tp if t is x else x for x in (q, k, v)]
            args_m = [tm if t is x else x for x in (q, k, v)]
            fd = (f(*args_p) - f(*args_m)) / (2 * e)
            assert abs(fd - grad[idx].item()) <= 2e-3 * max(1.0, abs(fd)), (causal, idx)
