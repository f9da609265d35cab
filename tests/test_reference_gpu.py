"""The reference's own GPU implementations, run on the same B200 as a second comparator.

The reference installs (``pip install --target baseline/_ref``, git-ignored) as its ``kernels``
package -- the fp16 Triton flash-attention forward (kernels/flash_attn/flash_attn_fwd.py:131-156),
the Triton int8 GEMM + dequant (kernels/int8_gemm/int8_gemm.py:98-138), the pure-torch
``quantize_symmetric`` (:146-161) -- and its RMSNorm+Linear dispatcher
(kernels/fused_rmsnorm_linear/fused_ops.py:45-68).  Its CUDA extension compiles for sm_100
but does not import: csrc/bindings.cpp:12 declares launch_fused_rmsnorm_linear with at::Half
pointers and csrc/fused_rmsnorm_linear.cu:105 defines it with half pointers, so the symbol is
undefined and the dispatcher runs its PyTorch path (cuBLAS on fp16).  Each is run on CUDA
tensors beside this library's kernel and the CPU oracle.  Skipped when baseline/_ref is not
there.
"""

import os
import sys

import numpy as np
import pytest
import torch

import llm_kernels
import oracle
from conftest import ROOT

REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kernels")), reason="reference not installed in baseline/_ref"),
]


@pytest.fixture(scope="module")
def ref():
    if REF not in sys.path:
        sys.path.append(REF)  # appended: this library's llm_kernels stays the one imported
    import kernels

    return kernels


def _err(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_reference_triton_flash_attention_and_ours_agree(ref, D, causal):
    g = torch.Generator().manual_seed(50 + D)
    q, k, v = (torch.randn(1, 4, 1024, D, generator=g).to(torch.float16).cuda() for _ in range(3))
    theirs = ref.flash_attn_forward(q, k, v, causal=causal)
    ours = llm_kernels.flash_attn_forward(q, k, v, causal=causal)
    exact = oracle.attention_fp32(q, k, v, causal)
    assert _err(theirs, exact) <= 1e-2
    assert _err(ours, exact) <= 1e-2
    assert _err(ours, theirs) <= 1e-2


def test_reference_triton_int8_gemm_bit_exact(ref):
    """Same int32 accumulator, same (fp32(acc) * sa) * sb epilogue: identical fp16 bits."""
    g = torch.Generator().manual_seed(51)
    A_q, sa = llm_kernels.quantize_symmetric(torch.randn(1024, 1024, generator=g).to(torch.float16).cuda())
    B_q, sb = llm_kernels.quantize_symmetric(torch.randn(768, 1024, generator=g).to(torch.float16).cuda())
    B_kn = B_q.T.contiguous()
    theirs = ref.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb)
    ours = llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb)
    assert torch.equal(theirs.view(torch.int16), ours.view(torch.int16))


def test_reference_quantize_on_cuda_vs_its_cpu_path(ref):
    """The reference's quantize_symmetric on CUDA tensors divides through torch's CUDA kernel
    for `tensor / scalar`; its CPU path (what this library and the oracle match bit for bit)
    uses an IEEE division.  Measured here: their CUDA scales equal the CPU ones or differ by
    one ulp, and a code differs by at most 1, only in rows whose scale differs or at a near
    tie."""
    g = torch.Generator().manual_seed(52)
    x = (torch.randn(512, 4096, generator=g) * 3).to(torch.float16)
    q_gpu, s_gpu = ref.quantize_symmetric(x.cuda())
    q_ours, s_ours = llm_kernels.quantize_symmetric(x.cuda())
    q_cpu, s_cpu = oracle.quantize_symmetric(x)
    assert np.array_equal(q_ours.cpu().numpy(), q_cpu) and np.array_equal(s_ours.cpu().numpy(), s_cpu)
    sg = s_gpu.float().cpu().numpy().view(np.int32).astype(np.int64)
    sc = s_cpu.view(np.int32).astype(np.int64)
    ulp = np.abs(sg - sc)
    dq = np.abs(q_gpu.cpu().numpy().astype(np.int32) - q_cpu.astype(np.int32))
    assert ulp.max() <= 1, ulp.max()
    assert dq.max() <= 1, dq.max()
    print(f"reference quantize on CUDA vs CPU: {int((ulp > 0).sum())}/{ulp.size} scales differ by 1 ulp, "
          f"{int((dq > 0).sum())}/{dq.size} codes differ by 1")


def test_reference_rmsnorm_linear_dispatcher_and_ours_agree(ref):
    g = torch.Generator().manual_seed(53)
    x = torch.randn(64, 1024, generator=g)
    w_norm = 1 + 0.1 * torch.randn(1024, generator=g)
    w_lin = torch.randn(512, 1024, generator=g) / 32
    exact = oracle.rmsnorm_linear_ref(x, w_norm, w_lin)
    xs, wn, wl = x.half().cuda(), w_norm.half().cuda(), w_lin.half().cuda()
    theirs = ref.fused_rmsnorm_linear(xs, wn, wl)
    ours = llm_kernels.fused_rmsnorm_linear(xs, wn, wl)
    scale = exact.abs().max().item()
    assert _err(theirs, exact) / scale <= 1e-2
    assert _err(ours, exact) / scale <= 1e-2
