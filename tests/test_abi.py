"""C-ABI checks that need no GPU: the library loads, exports exactly the header's entry
points, and rejects bad arguments on the host before touching CUDA."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from llm_kernels import _lib

HEADER = os.path.join(ROOT, "include", "llm_kernels_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"LK_API\s+[\w\s\*]+?\b(lk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    fns = header_functions()
    for f in ("lk_quantize_symmetric", "lk_int8_gemm_dequant", "lk_int8_gemm_i32", "lk_flash_attn_fwd",
              "lk_rmsnorm_linear_fold", "lk_rmsnorm_linear", "lk_fused_rmsnorm_linear"):
        assert f in fns


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_python_binding_covers_header():
    assert sorted(_lib.SIGNATURES) == header_functions()


def test_status_strings():
    lib = _lib.load()
    assert lib.lk_status_string(0) == b"ok"
    assert b"timed out" in lib.lk_status_string(_lib.LK_ERR_TIMEOUT)
    assert lib.lk_version() >> 16 == 1


def test_bad_arguments_rejected_on_host():
    lib = _lib.load()
    null = None
    # negative / null arguments fail before any CUDA call
    assert lib.lk_quantize_symmetric(null, _lib.LK_F16, 4, 8, 8, null, 8, null, null) == _lib.LK_ERR_INVALID_ARG
    assert lib.lk_quantize_symmetric(null, _lib.LK_F16, -1, 8, 8, null, 8, null, null) == _lib.LK_ERR_INVALID_ARG
    assert lib.lk_int8_gemm_dequant(null, 64, null, 64, 0, null, null, null, 64, 8, 8, 64, null) == _lib.LK_ERR_INVALID_ARG
    assert lib.lk_int8_gemm_i32(null, 64, null, 64, 7, null, 64, 8, 8, 64, null) == _lib.LK_ERR_INVALID_ARG
    s4 = _lib.i64_array([0, 0, 0, 1])
    assert lib.lk_flash_attn_fwd(null, null, null, null, _lib.LK_BF16, 1, 1, 16, 16, 128, s4, s4, s4, s4, 1, 0.0,
                                 null) == _lib.LK_ERR_INVALID_ARG
    assert lib.lk_rmsnorm_linear(null, 64, null, null, 64, _lib.LK_BF16, 4, 64, 64, 1e-6, null,
                                 null) == _lib.LK_ERR_INVALID_ARG
    # grouped-query: H_kv must divide H (checked before any pointer or device use)
    for h_kv in (0, -2, 3, 5):
        assert lib.lk_flash_attn_fwd_gqa(null, null, null, null, _lib.LK_BF16, 1, 8, h_kv, 16, 16, 128, s4, s4, s4, s4,
                                         1, 0.0, null) == _lib.LK_ERR_INVALID_ARG


def test_empty_work_is_a_noop():
    lib = _lib.load()
    assert lib.lk_quantize_symmetric(None, _lib.LK_F16, 0, 8, 8, None, 8, None, None) == _lib.LK_OK
    assert lib.lk_int8_gemm_dequant(None, 64, None, 64, 0, None, None, None, 64, 0, 8, 64, None) == _lib.LK_OK
