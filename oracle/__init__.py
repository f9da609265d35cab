"""CPU oracle for the llm_kernels inference op set — TEST INFRASTRUCTURE ONLY.

These functions restate the reference's algorithms on the CPU (numpy for the byte/integer
work, a small C library for the int32 GEMM, torch fp32 on CPU for the two floating-point
ops) and exist only to check the sm_100a kernels.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline / reference arm may import this package; the product path in
``llm_kernels`` never does.

Parity pin: every function here is checked against golden vectors produced by the reference
itself (its Python functions, and its Triton kernels run under ``TRITON_INTERPRET=1``) —
see ``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``.
"""

from .quantize import quantize_symmetric
from .int8_gemm import int8_gemm_i32, dequant_f16, int8_gemm_dequant
from .attention import attention_fp32, attention_gqa_fp32, attention_grad_fp32, attention_lse_fp32
from .rmsnorm_linear import rmsnorm_linear_ref

__all__ = [
    "quantize_symmetric",
    "int8_gemm_i32",
    "dequant_f16",
    "int8_gemm_dequant",
    "attention_fp32",
    "attention_gqa_fp32",
    "attention_grad_fp32",
    "attention_lse_fp32",
    "rmsnorm_linear_ref",
]
