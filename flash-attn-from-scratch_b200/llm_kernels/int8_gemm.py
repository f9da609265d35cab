"""int8 symmetric GEMM with fused dequantisation, and the per-row quantiser.

Drop-in for the reference's ``kernels/int8_gemm/int8_gemm.py``:
  * ``quantize_symmetric(x)`` — int8_gemm.py:146-161, bit-exact (codes and fp32 scales),
  * ``int8_gemm_dequant_fwd(A, B, scale_a, scale_b, block_m, block_n, block_k)`` — :98-138,
  * ``int8_gemm_dequant_auto`` — :192-200 (the tile heuristic; tiles are fixed here).
Both run sm_100a kernels through the C ABI: a warp-per-row quantiser and a tcgen05
``kind::i8`` GEMM whose int32 accumulator lives in tensor memory and is dequantised in the
epilogue, so it never reaches HBM.
"""

from __future__ import annotations

import torch

from . import _lib
from ._common import dtype_code, ptr, require, require_cuda, stream_for

__all__ = [
    "quantize_symmetric",
    "int8_gemm_dequant_fwd",
    "int8_gemm_dequant_auto",
    "int8_gemm_i32",
    "int8_gemm_dequant_nk",
    "int8_gemm_dequant_scatter",
    "int8_gemm_dequant_requant",
    "int8_gemm_dequant_multicast",
]


def quantize_symmetric(x: torch.Tensor):
    """Per-row symmetric absmax quantisation (int8_gemm.py:146-161).

    Args:
        x : [..., K] fp32 / fp16 / bf16, CUDA.

    Returns:
        x_q   : [..., K] int8, ``clamp(round(x / scale), -128, 127)``
        scale : [...]    fp32, ``amax(|x|, -1) / 127``
    """
    require_cuda("quantize_symmetric", x)
    require(x.dtype in (torch.float32, torch.float16, torch.bfloat16), f"quantize_symmetric: unsupported dtype {x.dtype}")
    require(x.dim() >= 1, "quantize_symmetric: x must have at least one dimension")
    K = x.shape[-1]
    require(K > 0, "quantize_symmetric: cannot reduce over an empty last dimension")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    q = torch.empty((rows, K), dtype=torch.int8, device=x.device)
    scale = torch.empty((rows,), dtype=torch.float32, device=x.device)
    if rows:
        s = stream_for(x.device)
        _lib.call(
            "lk_quantize_symmetric",
            ptr(x2), dtype_code(x2.dtype), rows, K, x2.stride(0) if rows > 1 else K, ptr(q), K, ptr(scale), s,
        )
    return q.reshape(*lead, K), scale.reshape(lead)


def _gemm_checks(A: torch.Tensor, B: torch.Tensor, kn_layout: bool):
    require(A.dtype == torch.int8, "A must be int8")
    require(B.dtype == torch.int8, "B must be int8")
    require(A.is_cuda and B.is_cuda, "Inputs must be on CUDA")
    require(A.is_contiguous() and B.is_contiguous(), "Inputs must be contiguous")
    require(A.dim() == 2 and B.dim() == 2, "A and B must be 2-D")
    M, K = A.shape
    if kn_layout:
        K2, N = B.shape
    else:
        N, K2 = B.shape
    require(K == K2, f"Inner dimension mismatch: A has K={K}, B has K={K2}")
    return M, N, K


def _run_gemm(A, B, b_layout, scale_a, scale_b, M, N, K, out_dtype):
    dev = require_cuda("int8_gemm", A, B)
    C = torch.empty((M, N), device=A.device, dtype=out_dtype)
    if M == 0 or N == 0:
        return C
    if K == 0:
        return C.zero_()
    # TMA needs 16-byte row strides.  Shapes that violate it are re-laid out here (a copy,
    # not a different compute path): K is zero-padded to a multiple of 16 (zeros add nothing
    # to the int32 sum), and a [K, N] B with N % 16 != 0 is transposed to its [N, K] form.
    if K % 16:
        Kp = (K + 15) // 16 * 16
        A = torch.nn.functional.pad(A, (0, Kp - K))
        B = torch.nn.functional.pad(B, (0, 0, 0, Kp - K)) if b_layout == 0 else torch.nn.functional.pad(B, (0, Kp - K))
        K = Kp
    if b_layout == 0 and N % 16:
        B = B.t().contiguous()
        b_layout = 1
    s = stream_for(dev)
    ldb = B.shape[1]
    if out_dtype == torch.int32:
        _lib.call("lk_int8_gemm_i32", ptr(A), K, ptr(B), ldb, b_layout, ptr(C), N, M, N, K, s)
    else:
        require_cuda("int8_gemm_dequant_fwd", scale_a, scale_b)
        require(scale_a.dtype == torch.float32 and scale_b.dtype == torch.float32, "scales must be fp32")
        require(scale_a.numel() == M and scale_b.numel() == N, "scale_a must have M and scale_b N elements")
        sa = scale_a.contiguous()
        sb = scale_b.contiguous()
        _lib.call(
            "lk_int8_gemm_dequant", ptr(A), K, ptr(B), ldb, b_layout, ptr(sa), ptr(sb), ptr(C), N, M, N, K, s
        )
    return C


def int8_gemm_dequant_fwd(
    A: torch.Tensor,  # [M, K] int8, CUDA
    B: torch.Tensor,  # [K, N] int8, CUDA
    scale_a: torch.Tensor,  # [M] fp32 (per row of A)
    scale_b: torch.Tensor,  # [N] fp32 (per column of B)
    block_m: int = 128,
    block_n: int = 128,
    block_k: int = 64,
) -> torch.Tensor:
    """int8 GEMM with fused per-channel dequantisation (int8_gemm.py:98-138).

    ``C[m, n] = fp16((fp32(sum_k A[m,k] B[k,n]) * scale_a[m]) * scale_b[n])``.
    The tile kwargs are accepted for signature compatibility; the sm_100a kernel uses its own
    fixed tcgen05 tiling.

    Returns:
        C : [M, N] fp16
    """
    for name, v in (("block_m", block_m), ("block_n", block_n), ("block_k", block_k)):
        require(isinstance(v, int) and v > 0, f"{name} must be a positive int")
    M, N, K = _gemm_checks(A, B, kn_layout=True)
    return _run_gemm(A, B, 0, scale_a, scale_b, M, N, K, torch.float16)


def int8_gemm_dequant_nk(A, B_nk, scale_a, scale_b) -> torch.Tensor:
    """Same GEMM with B stored as [N, K] (a weight's natural layout), so no transpose copy."""
    M, N, K = _gemm_checks(A, B_nk, kn_layout=False)
    return _run_gemm(A, B_nk, 1, scale_a, scale_b, M, N, K, torch.float16)


def int8_gemm_dequant_scatter(A, B_nk, scale_a, scale_b, dst_ptrs, ldc: int, col_offset: int) -> None:
    """``int8_gemm_dequant_nk(A, B_nk, ...)`` stored straight into several fp16 matrices.

    The ``[M, N]`` result goes to columns ``[col_offset, col_offset + N)`` of every
    destination (device addresses in ``dst_ptrs``, 1 to 8 of them, each an fp16 matrix with row
    pitch ``ldc`` elements, e.g. all ranks' replicated outputs of a column-sharded layer) in the
    same launch; nothing is returned.  K must be a multiple of 16, ``ldc`` and ``col_offset``
    multiples of 8 and every address 16-byte aligned.
    """
    M, N, K = _gemm_checks(A, B_nk, kn_layout=False)
    dev = require_cuda("int8_gemm_dequant_scatter", A, B_nk, scale_a, scale_b)
    require(K % 16 == 0, "K must be a multiple of 16")
    require(scale_a.dtype == torch.float32 and scale_b.dtype == torch.float32, "scales must be fp32")
    require(scale_a.numel() == M and scale_b.numel() == N, "scale_a must have M and scale_b N elements")
    require(1 <= len(dst_ptrs) <= 8, "1 to 8 destinations")
    require(ldc % 8 == 0 and col_offset % 8 == 0 and ldc >= col_offset + N, "ldc/col_offset must be multiples of 8 "
            "and the block must fit in ldc")
    if M == 0 or N == 0:
        return
    import ctypes

    dsts = (ctypes.c_void_p * len(dst_ptrs))(*[int(p) for p in dst_ptrs])
    _lib.call("lk_int8_gemm_dequant_scatter", ptr(A), K, ptr(B_nk), K, 1, ptr(scale_a.contiguous()),
              ptr(scale_b.contiguous()), dsts, len(dst_ptrs), ldc, col_offset, M, N, K, stream_for(dev))


def int8_gemm_dequant_requant(A, B, scale_a, scale_b, b_layout: str = "nk", return_output: bool = False):
    """``quantize_symmetric(int8_gemm_dequant(A, B, scale_a, scale_b))`` in one kernel.

    The int8 GEMM's epilogue rounds its dequantised output to fp16 exactly as
    ``int8_gemm_dequant_fwd`` does and quantises it per row for the next int8 layer, so the
    fp16 activation need not make a round trip through HBM (the reference ran
    ``Int8Linear`` -> ``quantize_symmetric`` as separate passes, llm_kernels/__init__.py:111-118).
    Codes and scales are bit-identical to the two-step result.

    Args:
        A : [M, K] int8; B : [N, K] int8 (``"nk"``, a weight) or [K, N] (``"kn"``);
        scale_a : [M] fp32; scale_b : [N] fp32.
        return_output : also return the fp16 ``C`` (written by the same kernel).

    Returns:
        (q [M, N] int8, scale [M] fp32), or (q, scale, C) with ``return_output``.
    """
    require(b_layout in ("kn", "nk"), "b_layout must be 'kn' or 'nk'")
    kn = b_layout == "kn"
    M, N, K = _gemm_checks(A, B, kn_layout=kn)
    dev = require_cuda("int8_gemm_dequant_requant", A, B, scale_a, scale_b)
    require(scale_a.dtype == torch.float32 and scale_b.dtype == torch.float32, "scales must be fp32")
    require(scale_a.numel() == M and scale_b.numel() == N, "scale_a must have M and scale_b N elements")
    require(K % 16 == 0 and N % 16 == 0, "int8_gemm_dequant_requant: K and N must be multiples of 16")
    q = torch.empty((M, N), dtype=torch.int8, device=A.device)
    qs = torch.empty((M,), dtype=torch.float32, device=A.device)
    C = torch.empty((M, N), dtype=torch.float16, device=A.device) if return_output else None
    if M and N:
        lib = _lib.load()
        ws = torch.empty((int(lib.lk_int8_gemm_requant_workspace_bytes(M)),), dtype=torch.uint8, device=A.device)
        _lib.call("lk_int8_gemm_dequant_requant", ptr(A), K, ptr(B), B.shape[1], 0 if kn else 1,
                  ptr(scale_a.contiguous()), ptr(scale_b.contiguous()), ptr(C) if C is not None else None, N,
                  ptr(q), N, ptr(qs), ptr(ws), M, N, K, stream_for(dev))
    return (q, qs, C) if return_output else (q, qs)


def int8_gemm_dequant_multicast(A, B_nk, scale_a, scale_b, multicast_ptr: int, ldc: int, col_offset: int) -> None:
    """``int8_gemm_dequant_nk(A, B_nk, ...)`` stored through an NVLink multicast address.

    ``multicast_ptr`` addresses a multicast object bound to every rank's fp16 ``[M, ldc]``
    output (row pitch ``ldc``); the ``[M, N]`` result goes to columns ``[col_offset,
    col_offset + N)`` of all of them with one ``multimem`` store per 16 bytes.  N must be a
    multiple of 32, ``ldc`` and ``col_offset`` multiples of 8, K a multiple of 16.
    """
    M, N, K = _gemm_checks(A, B_nk, kn_layout=False)
    dev = require_cuda("int8_gemm_dequant_multicast", A, B_nk, scale_a, scale_b)
    require(K % 16 == 0 and N % 32 == 0, "K must be a multiple of 16 and N of 32")
    require(scale_a.dtype == torch.float32 and scale_b.dtype == torch.float32, "scales must be fp32")
    require(scale_a.numel() == M and scale_b.numel() == N, "scale_a must have M and scale_b N elements")
    require(ldc % 8 == 0 and col_offset % 8 == 0 and ldc >= col_offset + N, "ldc/col_offset must be multiples of 8 "
            "and the block must fit in ldc")
    require(multicast_ptr != 0 and multicast_ptr % 16 == 0, "multicast_ptr must be a 16-byte aligned address")
    if M == 0 or N == 0:
        return
    _lib.call("lk_int8_gemm_dequant_multicast", ptr(A), K, ptr(B_nk), K, 1, ptr(scale_a.contiguous()),
              ptr(scale_b.contiguous()), multicast_ptr, ldc, col_offset, M, N, K, stream_for(dev))


def int8_gemm_i32(A: torch.Tensor, B: torch.Tensor, b_layout: str = "kn") -> torch.Tensor:
    """The raw int32 accumulator ``A @ B`` (B as [K,N] for ``"kn"``, [N,K] for ``"nk"``)."""
    require(b_layout in ("kn", "nk"), "b_layout must be 'kn' or 'nk'")
    kn = b_layout == "kn"
    M, N, K = _gemm_checks(A, B, kn_layout=kn)
    return _run_gemm(A, B, 0 if kn else 1, None, None, M, N, K, torch.int32)


def int8_gemm_dequant_auto(A, B, scale_a, scale_b):
    """The reference's size heuristic (int8_gemm.py:192-200); tiling is fixed on sm_100a."""
    M = A.shape[0]
    if M <= 1024:
        bm, bn, bk = 64, 64, 64
    else:
        bm, bn, bk = 128, 128, 64
    return int8_gemm_dequant_fwd(A, B, scale_a, scale_b, block_m=bm, block_n=bn, block_k=bk)
