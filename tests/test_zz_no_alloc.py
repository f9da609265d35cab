"""lk_rmsnorm_linear_noalloc: RMSNorm + Linear for callers that cannot allocate device memory
at call time (the scratch lives in a fixed array inside the library).

Called through the C ABI and compared with lk_rmsnorm_linear, the entry point that takes a
caller-allocated scratch buffer, on two calls in a row (the second call reuses the array the
first one filled), within the tolerance of the other tests (and bit for bit where both take
the same kernels), and with the fp32 oracle.  The file's name makes pytest collect it last.
"""

import pytest
import torch

from llm_kernels import _lib

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2  # the RMSNorm+Linear tolerance of the other tests


def _inputs(rows, d_in, d_out, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, d_in, generator=g).to(torch.bfloat16).cuda()
    w_norm = (1 + 0.1 * torch.randn(d_in, generator=g)).to(torch.bfloat16).cuda()
    w_lin = (torch.randn(d_out, d_in, generator=g) / d_in ** 0.5).to(torch.bfloat16).cuda()
    return x, w_norm, w_lin


def _fold(w_norm, w_lin, stream):
    w_fold = torch.empty_like(w_lin)
    d_out, d_in = w_lin.shape
    _lib.call("lk_rmsnorm_linear_fold", w_norm.data_ptr(), _lib.LK_BF16, w_lin.data_ptr(), w_fold.data_ptr(),
              _lib.LK_BF16, d_in, d_out, stream)
    return w_fold


def _with_scratch(x, w_fold, eps, stream):
    rows, d_in = x.shape
    d_out = w_fold.shape[0]
    y = torch.empty(rows, d_out, dtype=x.dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.call("lk_rmsnorm_linear", x.data_ptr(), d_in, w_fold.data_ptr(), y.data_ptr(), d_out, _lib.LK_BF16,
              rows, d_in, d_out, eps, rstd.data_ptr(), stream)
    return y


def _no_alloc(x, w_fold, eps, stream):
    rows, d_in = x.shape
    d_out = w_fold.shape[0]
    y = torch.empty(rows, d_out, dtype=x.dtype, device=x.device)
    _lib.call("lk_rmsnorm_linear_noalloc", x.data_ptr(), d_in, w_fold.data_ptr(), y.data_ptr(), d_out,
              _lib.LK_BF16, rows, d_in, d_out, eps, stream)
    return y


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


def test_no_alloc_matches_scratch_entry_point_twice():
    _lib.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    # Call 1 fills more rows of the shared array than call 2 reads; call 2 must not see them.
    for rows, d_in, d_out, seed in ((1000, 1024, 768, 1), (300, 512, 1024, 2)):
        x, w_norm, w_lin = _inputs(rows, d_in, d_out, seed)
        w_fold = _fold(w_norm, w_lin, stream)
        ref = _with_scratch(x, w_fold, 1e-6, stream)
        out = _no_alloc(x, w_fold, 1e-6, stream)
        torch.cuda.synchronize()
        assert _rel(out, ref) <= REL_TOL
        assert torch.equal(out, ref)  # these problems take the same kernels on both entry points


def test_no_alloc_rejects_rows_beyond_the_fixed_scratch():
    lib = _lib.load()
    st = lib.lk_rmsnorm_linear_noalloc(None, 64, None, None, 64, _lib.LK_BF16, 65537, 64, 64, 1e-6, None)
    assert st == _lib.LK_ERR_SCRATCH_LIMIT
    assert b"65536" in lib.lk_status_string(st)


def test_no_alloc_allocates_nothing_on_the_pair_path():
    """2304 x 1024 -> 2304 runs on the CTA-pair GEMM, whose split tail would take a per-stream
    workspace on the entry point with caller scratch; the no-allocation entry point must leave
    device memory untouched, on a stream it has never seen."""
    _lib.set_device(0)
    x, w_norm, w_lin = _inputs(2304, 1024, 2304, 3)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        w_fold = _fold(w_norm, w_lin, side.cuda_stream)
        y = torch.empty(2304, 2304, dtype=x.dtype, device=x.device)
        y.zero_()  # the stream's first kernel: any lazy per-stream set-up happens here
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    _lib.call("lk_rmsnorm_linear_noalloc", x.data_ptr(), 1024, w_fold.data_ptr(), y.data_ptr(), 2304,
              _lib.LK_BF16, 2304, 1024, 2304, 1e-6, side.cuda_stream)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    ref = _with_scratch(x, w_fold, 1e-6, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _rel(y, ref) <= REL_TOL
    # and directly against the fp32 oracle of the reference's op (fused_ops.py:27-37)
    import oracle

    exact = oracle.rmsnorm_linear_ref(x.float().cpu(), w_norm.float().cpu(), w_lin.float().cpu())
    assert _rel(y.cpu(), exact) <= REL_TOL
