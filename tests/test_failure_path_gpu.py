"""The device failure path: a bounded wait that runs out is reported, the kernel unwinds, and
the context stays usable.

The reference has no device-side error path (kernels/flash_attn/flash_attn_fwd.py:132-135 only
asserts on the host); this library's kernels never trap: every pipeline wait is bounded, and a
wait that runs out records (LK_ERR_TIMEOUT, site, block, thread) in a device status word, after
which every role drains the copies and MMAs it started, frees tensor memory and returns.

Each test arms a one-shot test hook (lk_debug_inject) that withholds ONE copy or ONE counter
update in a tiny launch, so a consumer's wait cannot complete; the wait limit is lowered to
20 ms for the duration (lk_debug_set_wait_limit).  Nothing faults or hangs: the launch returns
within a few wait limits with the status set.  The test then checks the status word, clears it
and runs the same problem again on the same stream, which must match the oracle exactly as a
normal launch does.
"""

import contextlib

import numpy as np
import pytest
import torch

import llm_kernels
import oracle
from llm_kernels import _lib

pytestmark = pytest.mark.gpu

LIMIT_NS = 20_000_000  # 20 ms: far above any legitimate wait of these tiny launches

FA_SITES = range(201, 209)     # csrc/flash_attn.cu Site
GEMM_SITES = range(101, 107)   # csrc/gemm_sm100.cuh Site
PAIR_SPLIT_SITE = 126          # csrc/gemm_pair_sm100.cuh kSitePairSplit
PAIR_REQUANT_SITE = 127        # csrc/gemm_pair_sm100.cuh kSitePairRequant


@contextlib.contextmanager
def short_waits():
    _lib.set_device(torch.cuda.current_device())
    _lib.call("lk_debug_set_wait_limit", LIMIT_NS)
    try:
        yield
    finally:
        _lib.call("lk_debug_inject", _lib.LK_INJECT_NONE, 0, 0)
        _lib.call("lk_debug_set_wait_limit", 0)


def _expect_timeout(sites):
    code, site, blk, thr = llm_kernels.device_status()
    assert code == _lib.LK_ERR_TIMEOUT, (code, site, blk, thr)
    assert site in sites, site
    llm_kernels.clear_device_status()
    assert llm_kernels.device_status() == (0, 0, 0, 0)
    return blk


@pytest.mark.parametrize("item", [0, 3])
def test_flash_attention_lost_load_times_out_and_recovers(item):
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(1, 1, 256, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    with short_waits():
        _lib.call("lk_debug_inject", _lib.LK_INJECT_FA_DROP_LOAD, 0, item)  # item 0 = K_0, 3 = V_1
        llm_kernels.flash_attn_forward(q, k, v, causal=False)
        assert _expect_timeout(FA_SITES) == 0
    ref = oracle.attention_fp32(q, k, v, False)
    out = llm_kernels.flash_attn_forward(q, k, v, causal=False)
    assert (out.float().cpu() - ref).abs().max().item() <= 1e-2


def test_one_cta_gemm_lost_load_times_out_and_recovers():
    g = torch.Generator().manual_seed(12)
    A = torch.randint(-128, 128, (256, 512), generator=g, dtype=torch.int8).cuda()
    B = torch.randint(-128, 128, (256, 512), generator=g, dtype=torch.int8).cuda()  # [N, K]
    ref = oracle.int8_gemm_i32(A.cpu().numpy(), B.cpu().numpy(), "nk")
    with short_waits():
        # 256 x 256 x 512 runs on the one-CTA kernel (4 CTAs of 128 x 128, 4 stages each)
        _lib.call("lk_debug_inject", _lib.LK_INJECT_GEMM_DROP_LOAD, 1, 2)
        llm_kernels.int8_gemm_i32(A, B, "nk")
        assert _expect_timeout(GEMM_SITES) == 1
    np.testing.assert_array_equal(llm_kernels.int8_gemm_i32(A, B, "nk").cpu().numpy(), ref)


def test_split_tail_lost_partial_times_out_and_clear_rearms_the_workspace():
    """A split-tail finisher whose writer never publishes gives up, leaving its tile's arrival
    counter set in the stream's workspace; clearing the status re-zeroes the workspace, so the
    next split launches on the same stream are bit-exact again."""
    M, N, K = 2200, 2144, 2048  # 81 tiles on 74 SM pairs: 7 leftover tiles split in 2 along K
    g = torch.Generator().manual_seed(13)
    A = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    B = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    ref = oracle.int8_gemm_i32(A.numpy(), B.numpy(), "nk")
    Ad, Bd = A.cuda(), B.cuda()
    np.testing.assert_array_equal(llm_kernels.int8_gemm_i32(Ad, Bd, "nk").cpu().numpy(), ref)
    with short_waits():
        _lib.call("lk_debug_inject", _lib.LK_INJECT_SPLIT_SKIP_PUBLISH, 0, 0)
        llm_kernels.int8_gemm_i32(Ad, Bd, "nk")
        _expect_timeout({PAIR_SPLIT_SITE})
    for _ in range(2):
        np.testing.assert_array_equal(llm_kernels.int8_gemm_i32(Ad, Bd, "nk").cpu().numpy(), ref)


def test_injection_is_one_shot_and_validated():
    lib = _lib.load()
    assert lib.lk_debug_inject(99, 0, 0) == _lib.LK_ERR_INVALID_ARG
    assert lib.lk_debug_inject(_lib.LK_INJECT_FA_DROP_LOAD, -1, 0) == _lib.LK_ERR_INVALID_ARG
    # armed for the GEMM, so a flash-attention launch does not take it
    try:
        _lib.call("lk_debug_inject", _lib.LK_INJECT_GEMM_DROP_LOAD, 0, 0)
        q = torch.randn(1, 1, 128, 64, dtype=torch.float16, device="cuda")
        llm_kernels.flash_attn_forward(q, q, q)
        assert llm_kernels.device_status()[0] == 0
    finally:
        _lib.call("lk_debug_inject", _lib.LK_INJECT_NONE, 0, 0)


def test_requant_unpublished_row_block_times_out_and_recovers():
    """The re-quantising GEMM's codes warps wait for every tile of their row block to publish its
    row maxima.  One epilogue warp that never publishes makes that wait run out: the launch
    reports LK_ERR_TIMEOUT at the requant site and unwinds, and the next call (which clears its
    workspace itself) is bit-exact again."""
    M, N, K = 512, 768, 256  # 2 x 3 pair tiles
    g = torch.Generator().manual_seed(14)
    A = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    W = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    sa = torch.rand(M, generator=g) * 1e-3
    sw = torch.rand(N, generator=g) * 1e-3
    ref_c = oracle.int8_gemm_dequant(A.numpy(), W.numpy(), sa.numpy(), sw.numpy(), "nk")
    rq, rs = oracle.quantize_symmetric(torch.from_numpy(ref_c))
    Ad, Wd, sad, swd = A.cuda(), W.cuda(), sa.cuda(), sw.cuda()
    with short_waits():
        _lib.call("lk_debug_inject", _lib.LK_INJECT_REQUANT_SKIP_PUBLISH, 1, 0)
        llm_kernels.int8_gemm_dequant_requant(Ad, Wd, sad, swd, "nk")
        _expect_timeout({PAIR_REQUANT_SITE})
    for _ in range(2):
        q, s = llm_kernels.int8_gemm_dequant_requant(Ad, Wd, sad, swd, "nk")
        np.testing.assert_array_equal(q.cpu().numpy(), rq)
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
