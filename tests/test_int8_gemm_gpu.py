"""int8 GEMM on the GPU vs the oracle: bit-exact int32 accumulator and bit-exact fp16
dequantised output, both B layouts, ragged shapes, and the 4096^3 config."""

import os

import numpy as np
import pytest
import torch

import llm_kernels
import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _rand_i8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


SHAPES = [(128, 256, 128), (256, 512, 384), (100, 72, 96), (1, 16, 16), (129, 257, 144), (300, 1000, 512),
          (1024, 1024, 1024), (64, 4096, 4096), (17, 40, 50), (3, 5, 7),
          # enough 256x256 tiles for the CTA-pair kernel, with ragged edges
          (2200, 2144, 512), (2304, 2304, 384), (4100, 3000, 200)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_int32_accumulator_bit_exact(M, N, K, layout):
    A = _rand_i8((M, K), 1 + M)
    B = _rand_i8((K, N) if layout == "kn" else (N, K), 2 + N)
    C = llm_kernels.int8_gemm_i32(A.cuda(), B.cuda(), layout)
    ref = oracle.int8_gemm_i32(A.numpy(), B.numpy(), layout)
    np.testing.assert_array_equal(C.cpu().numpy(), ref)


# (2304, 2300, *): CTA-pair kernel with a C row pitch that is not a multiple of 16 bytes, so C
# is stored directly instead of through TMA tiles (unsplit, and split 4 ways along K).
@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (100, 72, 96), (512, 512, 512), (333, 160, 256), (2200, 2144, 512),
                                   (2304, 2300, 1024), (2304, 2300, 4096)])
def test_dequant_fp16_bit_exact(M, N, K):
    g = torch.Generator().manual_seed(7 + M)
    A_fp = torch.randn(M, K, generator=g).to(torch.float16)
    B_fp = torch.randn(K, N, generator=g).to(torch.float16)
    A_q, sa = llm_kernels.quantize_symmetric(A_fp.cuda())
    B_q, sb = llm_kernels.quantize_symmetric(B_fp.T.contiguous().cuda())
    B_kn = B_q.T.contiguous()
    C = llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb)
    ref = oracle.int8_gemm_dequant(A_q.cpu().numpy(), B_kn.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy(), "kn")
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    C2 = llm_kernels.int8_gemm_dequant_nk(A_q, B_q, sa, sb)
    np.testing.assert_array_equal(C2.cpu().numpy().view(np.uint16), ref.view(np.uint16))


# Shapes whose leftover 256x256 tiles the CTA-pair kernel splits along K into 2, 3 and 4 parts
# (7, 23 and 7 left over of 81, 171 and 81 tiles on 74 pairs), with ragged edges.
SPLIT_SHAPES = [(2200, 2144, 2048), (2304, 4864, 3072), (2200, 2144, 4096)]


@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_split_tail_bit_exact(M, N, K, layout):
    A = _rand_i8((M, K), 11 + M)
    B = _rand_i8((K, N) if layout == "kn" else (N, K), 12 + N)
    Ad, Bd = A.cuda(), B.cuda()
    ref = oracle.int8_gemm_i32(A.numpy(), B.numpy(), layout)
    C = llm_kernels.int8_gemm_i32(Ad, Bd, layout)
    np.testing.assert_array_equal(C.cpu().numpy(), ref)
    # the split counters are re-armed by each launch: a second launch on the same stream, after
    # one of another shape, and one on a side stream agree bit for bit
    llm_kernels.int8_gemm_i32(Ad[:, : K // 2].contiguous(), Bd[: K // 2].contiguous() if layout == "kn"
                              else Bd[:, : K // 2].contiguous(), layout)
    C2 = llm_kernels.int8_gemm_i32(Ad, Bd, layout)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        C3 = llm_kernels.int8_gemm_i32(Ad, Bd, layout)
    torch.cuda.current_stream().wait_stream(side)
    assert torch.equal(C2, C) and torch.equal(C3, C)


def test_split_tail_dequant_fp16_bit_exact():
    M, N, K = 2304, 4864, 3072
    g = torch.Generator().manual_seed(21)
    A_q, sa = llm_kernels.quantize_symmetric(torch.randn(M, K, generator=g).to(torch.float16).cuda())
    B_q, sb = llm_kernels.quantize_symmetric(torch.randn(N, K, generator=g).to(torch.float16).cuda())
    ref = oracle.int8_gemm_dequant(A_q.cpu().numpy(), B_q.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy(), "nk")
    C = llm_kernels.int8_gemm_dequant_nk(A_q, B_q, sa, sb)
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    C_kn = llm_kernels.int8_gemm_dequant_fwd(A_q, B_q.T.contiguous(), sa, sb)
    np.testing.assert_array_equal(C_kn.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_golden_vectors_from_reference_kernel():
    g = np.load(os.path.join(GOLDEN, "int8_gemm.npz"))
    for tag in ("sq", "rag"):
        A = torch.from_numpy(g[f"{tag}_A"]).cuda()
        B = torch.from_numpy(g[f"{tag}_B_kn"]).cuda()
        sa = torch.from_numpy(g[f"{tag}_sa"]).cuda()
        sb = torch.from_numpy(g[f"{tag}_sb"]).cuda()
        C = llm_kernels.int8_gemm_dequant_fwd(A, B, sa, sb)
        np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), g[f"{tag}_C"].view(np.uint16))


def test_full_size_4096_cubed():
    """Config 3: M=N=K=4096, inputs quantised per row.  The accumulator of a row block is
    checked bit-exactly against the oracle and the whole matrix through an exact checksum
    (sum over n of C[m,n] == A[m,:] . rowsum(B)), computed in int64."""
    g = torch.Generator().manual_seed(2)
    A_fp = torch.randn(4096, 4096, generator=g).to(torch.float16)
    B_fp = torch.randn(4096, 4096, generator=g).to(torch.float16)  # [N, K]
    A_q, sa = llm_kernels.quantize_symmetric(A_fp.cuda())
    B_q, sb = llm_kernels.quantize_symmetric(B_fp.cuda())
    B_kn = B_q.T.contiguous()
    acc = llm_kernels.int8_gemm_i32(A_q, B_kn, "kn")
    rows = slice(1024, 1280)
    ref = oracle.int8_gemm_i32(A_q[rows].cpu().numpy(), B_q.cpu().numpy(), "nk")
    np.testing.assert_array_equal(acc[rows].cpu().numpy(), ref)
    # the 34 tiles left over after 3 rounds of 74 pairs (split along K): M-blocks 14-15 from
    # N-block 11, M-blocks 8-15 of N-blocks 12-15, all inside rows 2048.. and columns 2816..
    ref_tail = oracle.int8_gemm_i32(A_q[2048:].cpu().numpy(), B_q[2816:].cpu().numpy(), "nk")
    np.testing.assert_array_equal(acc[2048:, 2816:].cpu().numpy(), ref_tail)
    lhs = acc.to(torch.int64).sum(1)
    rhs = (A_q.to(torch.int64) * B_q.to(torch.int64).sum(0)[None, :]).sum(1)
    assert torch.equal(lhs, rhs)
    col_lhs = acc.to(torch.int64).sum(0)
    col_rhs = (B_q.to(torch.int64) * A_q.to(torch.int64).sum(0)[None, :]).sum(1)
    assert torch.equal(col_lhs, col_rhs)
    C = llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb)
    refC = oracle.dequant_f16(acc.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy())
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), refC.view(np.uint16))


def test_int8_linear_module_matches_oracle():
    torch.manual_seed(6)
    layer = llm_kernels.Int8Linear(256, 384)
    w = torch.randn(384, 256, dtype=torch.float16).cuda()
    layer.quantize_weights(w)
    x = torch.randn(40, 256, dtype=torch.float16).cuda()
    y = layer(x)
    xq, sx = oracle.quantize_symmetric(x.cpu())
    ref = oracle.int8_gemm_dequant(xq, layer.w_q.cpu().numpy(), sx, layer.scale_w.cpu().numpy(), "nk")
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("M", [512, 1024, 1025, 2304])
def test_auto_tile_heuristic_entry_point(M):
    """int8_gemm_dequant_auto (kernels/int8_gemm/int8_gemm.py:192-200) picks 64^3 tiles for
    M <= 1024 and 128x128x64 above; here both branches reach the same sm_100a GEMM and must
    equal the oracle bit for bit (M = 2304 also takes the CTA-pair kernel)."""
    N, K = 2304, 512
    g = torch.Generator().manual_seed(31 + M)
    A_q, sa = llm_kernels.quantize_symmetric(torch.randn(M, K, generator=g).to(torch.float16).cuda())
    B_q, sb = llm_kernels.quantize_symmetric(torch.randn(N, K, generator=g).to(torch.float16).cuda())
    B_kn = B_q.T.contiguous()
    C = llm_kernels.int8_gemm_dequant_auto(A_q, B_kn, sa, sb)
    ref = oracle.int8_gemm_dequant(A_q.cpu().numpy(), B_kn.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy(), "kn")
    assert C.shape == (M, N) and C.dtype == torch.float16
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_zero_and_degenerate_shapes():
    A = torch.zeros(0, 64, dtype=torch.int8, device="cuda")
    B = torch.zeros(64, 32, dtype=torch.int8, device="cuda")
    out = llm_kernels.int8_gemm_dequant_fwd(A, B, torch.ones(0, device="cuda"), torch.ones(32, device="cuda"))
    assert out.shape == (0, 32) and out.dtype == torch.float16


# Scatter epilogue (the column-sharded layer's fused gather), on one GPU: the column block is
# stored into two destination matrices at a column offset; both must equal the plain GEMM's
# result bit for bit and the columns outside the block must stay untouched.  Shapes reach the
# 1-CTA kernel (small), the CTA-pair kernel (2304 x 2048) and its split tail (4096 x 2048).
@pytest.mark.parametrize("M,N,K,col0,ldc", [(300, 200, 256, 8, 512), (128, 256, 128, 0, 256), (2304, 2048, 512, 1024, 4096),
                                             (4096, 2048, 4096, 2048, 4096), (77, 40, 48, 16, 64)])
def test_scatter_epilogue_matches_plain_gemm(M, N, K, col0, ldc):
    from llm_kernels.int8_gemm import int8_gemm_dequant_scatter

    g = torch.Generator().manual_seed(M + N)
    A = _rand_i8((M, K), 3 + M).cuda()
    B = _rand_i8((N, K), 4 + N).cuda()
    sa = (torch.rand(M, generator=g) * 0.02 + 1e-3).cuda()
    sb = (torch.rand(N, generator=g) * 0.02 + 1e-3).cuda()
    ref = llm_kernels.int8_gemm_dequant_nk(A, B, sa, sb)
    dsts = [torch.full((M, ldc), 7.0, dtype=torch.float16, device="cuda") for _ in range(2)]
    for _ in range(2):  # twice: the second launch must not depend on the first
        int8_gemm_dequant_scatter(A, B, sa, sb, [d.data_ptr() for d in dsts], ldc, col0)
    for d in dsts:
        assert torch.equal(d[:, col0:col0 + N], ref)
        outside = torch.cat([d[:, :col0], d[:, col0 + N:]], 1)
        assert bool((outside == 7.0).all())


def test_dequant_into_unaligned_output_through_the_c_abi():
    """A C-ABI caller may pass an output that is only 2-byte aligned (here one fp16 element
    into a buffer): the epilogue falls back to element stores instead of 16-byte ones."""
    from llm_kernels import _lib
    from llm_kernels._common import ptr, stream_for

    M, N, K = 2304, 2304, 256  # CTA-pair kernel (C base not 16-byte aligned: no TMA store)
    A = _rand_i8((M, K), 11).cuda()
    B = _rand_i8((N, K), 12).cuda()
    sa = torch.full((M,), 0.01, device="cuda")
    sb = torch.full((N,), 0.02, device="cuda")
    ref = llm_kernels.int8_gemm_dequant_nk(A, B, sa, sb)
    for m, n in ((M, N), (200, 300)):  # and the 1-CTA kernel
        buf = torch.zeros(m * N + 8, dtype=torch.float16, device="cuda")
        out = buf[1:1 + m * N].view(m, N)
        assert out.data_ptr() % 16 == 2
        _lib.call("lk_int8_gemm_dequant", ptr(A[:m]), K, ptr(B[:n]), K, 1, ptr(sa[:m]), ptr(sb[:n]), ptr(out), N,
                  m, n, K, stream_for(A.device))
        assert torch.equal(out[:, :n], ref[:m, :n])


# GEMM + dequant + re-quantisation of the fp16 output in one kernel (the O projection feeding
# the next int8 layer): codes and scales must equal quantize_symmetric of the plain GEMM's
# output bit for bit, C too when it is written.  Shapes: one tile; ragged M and N; N = 11008
# (43 tiles per row block, rounds that straddle row blocks); config 5's 4096-wide O projection
# with K = 4096; a few rows only.
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (300, 1008, 256), (1000, 11008, 512), (4096, 4096, 4096),
                                   (8, 512, 64), (2304, 2304, 1024)])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_requant_epilogue_matches_quantize_of_output(M, N, K, layout):
    g = torch.Generator().manual_seed(M * 7 + N)
    A_q, sa = llm_kernels.quantize_symmetric(torch.randn(M, K, generator=g).to(torch.float16).cuda())
    W_q, sw = llm_kernels.quantize_symmetric(torch.randn(N, K, generator=g).to(torch.float16).cuda())
    sa = sa * 0.25  # keep |C| well inside fp16 but over several binades
    B = W_q if layout == "nk" else W_q.T.contiguous()
    for _ in range(2):  # the second call must not see the first one's row maxima
        q, s, C = llm_kernels.int8_gemm_dequant_requant(A_q, B, sa, sw, layout, return_output=True)
    ref_c = oracle.int8_gemm_dequant(A_q.cpu().numpy(), W_q.cpu().numpy(), sa.cpu().numpy(), sw.cpu().numpy(), "nk")
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), ref_c.view(np.uint16))
    rq, rs = oracle.quantize_symmetric(torch.from_numpy(ref_c))
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    q2, s2 = llm_kernels.int8_gemm_dequant_requant(A_q, B, sa, sw, layout)
    assert torch.equal(q2, q) and torch.equal(s2, s)
    assert llm_kernels.device_status()[0] == 0


def test_requant_epilogue_special_rows():
    """Rows that overflow fp16 (scale inf: codes 0 where the quotient is NaN) and all-zero rows
    (scale 0, codes 0), as quantize_symmetric treats them."""
    M, N, K = 512, 768, 128
    A = _rand_i8((M, K), 21)
    A[3] = 0
    A[5] = 127
    W = _rand_i8((N, K), 22)
    W[:, :] = W.clamp(min=0)
    sa = torch.full((M,), 1e-3)
    sa[5] = 100.0  # row 5: 127 * 127 * K * 100 * sb overflows fp16
    sw = torch.full((N,), 1e-3)
    q, s, C = llm_kernels.int8_gemm_dequant_requant(A.cuda(), W.cuda(), sa.cuda(), sw.cuda(), "nk", return_output=True)
    ref_c = oracle.int8_gemm_dequant(A.numpy(), W.numpy(), sa.numpy(), sw.numpy(), "nk")
    assert np.isinf(ref_c[5].astype(np.float32)).any()
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint16), ref_c.view(np.uint16))
    rq, rs = oracle.quantize_symmetric(torch.from_numpy(ref_c))
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


def test_requant_rejects_too_wide_rows():
    from llm_kernels._lib import LKError

    A = torch.zeros(256, 64, dtype=torch.int8, device="cuda")
    W = torch.zeros(256 * 80, 64, dtype=torch.int8, device="cuda")
    with pytest.raises(LKError):
        llm_kernels.int8_gemm_dequant_requant(A, W, torch.ones(256, device="cuda"), torch.ones(256 * 80, device="cuda"))
