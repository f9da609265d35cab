"""quantize_symmetric on the GPU vs the oracle: bit-exact int8 codes and fp32 scales."""

import os

import numpy as np
import pytest
import torch

import llm_kernels
import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _check(x: torch.Tensor):
    q, s = llm_kernels.quantize_symmetric(x)
    assert q.dtype == torch.int8 and s.dtype == torch.float32
    assert q.shape == x.shape and s.shape == x.shape[:-1]
    rq, rs = oracle.quantize_symmetric(x.cpu())
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    gs = s.cpu().numpy()
    assert np.array_equal(np.isnan(gs), np.isnan(rs))
    ok = ~np.isnan(rs)
    assert np.array_equal(gs[ok].view(np.uint32), rs[ok].view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 8), (37, 200), (64, 4096), (5, 8192), (3, 12000), (7, 33), (2, 50000)])
def test_quantize_matches_oracle(dtype, shape):
    g = torch.Generator().manual_seed(hash((str(dtype), shape)) & 0xFFFF)
    x = (torch.randn(*shape, generator=g) * 2.5).to(dtype).cuda()
    _check(x)


def test_quantize_golden_vectors():
    g = np.load(os.path.join(GOLDEN, "quantize.npz"))
    for case in ("f16", "f32", "bf16", "f16_wide", "f32_special"):
        x = g[f"{case}_x"]
        xt = torch.from_numpy(x.astype(np.int16)).view(torch.bfloat16) if case == "bf16" else torch.from_numpy(x)
        q, s = llm_kernels.quantize_symmetric(xt.cuda())
        np.testing.assert_array_equal(q.cpu().numpy(), g[f"{case}_q"])
        ref_s = g[f"{case}_scale"]
        gs = s.cpu().numpy()
        assert np.array_equal(np.isnan(gs), np.isnan(ref_s))
        ok = ~np.isnan(ref_s)
        assert np.array_equal(gs[ok].view(np.uint32), ref_s[ok].view(np.uint32))


def test_quantize_special_rows():
    x = torch.randn(8, 64)
    x[0] = 0.0
    x[1, 7] = float("inf")
    x[2, 9] = float("nan")
    x[3] = -0.0
    x[4, :] = 1e-45
    x[5, 0] = -float("inf")
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        _check(x.to(dt).cuda())


def test_quantize_near_ties_take_the_exact_path():
    """Rows built so that many x / scale land exactly on, or within an ulp of, k + 0.5: the
    reciprocal fast path must hand those to the IEEE division and still match bit for bit."""
    rows = []
    g = torch.Generator().manual_seed(17)
    for a in (1.0, 0.37, 3.0e-3, 1.7e4, 1.1754944e-38 * 512):
        base = torch.arange(-127, 127, dtype=torch.float64) + 0.5
        jitter = torch.tensor([-1, 0, 1], dtype=torch.float64)
        vals = (base[:, None] * (1 + jitter[None, :] * 2.0 ** -23)).flatten()
        row = torch.cat([torch.tensor([127.0], dtype=torch.float64), vals])[:768] * a
        rows.append(row.float())
    x = torch.stack(rows)
    x = x[:, torch.randperm(x.shape[1], generator=g)]
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        _check(x.to(dt).cuda())
        _check(x.to(dt).repeat(1, 8).cuda())  # wide-row (CTA-per-row) kernels


def test_quantize_strided_rows_and_leading_dims():
    base = torch.randn(16, 300, dtype=torch.float16).cuda()
    _check(base[:, :256])  # row stride 300 != cols
    x3 = torch.randn(2, 5, 96, dtype=torch.bfloat16).cuda()
    q, s = llm_kernels.quantize_symmetric(x3)
    rq, rs = oracle.quantize_symmetric(x3.cpu())
    assert q.shape == (2, 5, 96) and s.shape == (2, 5)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


def test_quantize_full_size_4096sq():
    """The int8 GEMM config's operand (4096 x 4096 fp16): bit-exact against the oracle."""
    g = torch.Generator().manual_seed(2)
    x = torch.randn(4096, 4096, generator=g).to(torch.float16).cuda()
    _check(x)


def test_quantize_empty_rows():
    q, s = llm_kernels.quantize_symmetric(torch.empty(0, 64, device="cuda", dtype=torch.float16))
    assert q.shape == (0, 64) and s.shape == (0,)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_quantize_many_rows_specials_and_strides(dtype):
    """Thousands of 1024-wide rows (many waves of CTAs), fewer rows than SMs, rows holding
    zeros / inf / NaN / subnormals, and a row stride larger than the row."""
    g = torch.Generator().manual_seed(41)
    x = (torch.randn(6000, 1024, generator=g) * 3).to(dtype)
    x[5] = 0.0
    x[77, 3] = float("inf")
    x[1000, 9] = float("nan")
    x[4321, :] = 1e-40 if dtype == torch.float32 else 0.0
    x[5999, 100] = -float("inf")
    _check(x.cuda())
    _check(x[:100].cuda())
    wide = (torch.randn(40, 3000, generator=g) * 0.01).to(dtype).cuda()
    _check(wide[:, :2048])  # row stride 3000 elements, 16-byte multiple for every dtype
