"""CPU check of the flash-attention forward's FMA-pipe exponential (`exp2_poly_pair` in
csrc/fa_common.cuh).

The kernel computes one key pair in eight as 2^x without the MUFU unit: Cody-Waite reduction
x = rint(x) + f with the 1.5 * 2^23 shifter, a cubic for 2^f on [-1/2, 1/2], and rint(x)
added into the exponent field.  This test reads the four coefficients out of the header, redoes
the same float32 steps in numpy (each FMA rounded once, as `fma.rn.f32x2` does) and checks the
result against 2^x: relative error within the fitted bound over the whole input range the
softmax produces (scores minus the running maximum, at most +8 with lazy rescaling), and the
masked-key input (-inf) mapped to (about) 2^-125.
"""

import os
import re

import numpy as np

from conftest import PKG

HEADER = os.path.join(PKG, "csrc", "fa_common.cuh")


def _coefficients():
    src = open(HEADER).read()
    body = src[src.index("void exp2_poly_pair"):]
    body = body[: body.index("\n}\n")]
    # Horner order in the source: c3 (first fma's a), c2, c1, c0.
    lits = re.findall(r"lk::f2\((0x[0-9a-fA-F.]+p[-+]?\d+)f,", body)
    vals = []
    for lit in lits:
        v = np.float32(float.fromhex(lit))
        if not vals or vals[-1] != v:
            vals.append(v)
    assert len(vals) == 4, lits
    c3, c2, c1, c0 = vals
    return c0, c1, c2, c3


def _exp2_poly(x):
    c0, c1, c2, c3 = _coefficients()
    x = np.asarray(x, dtype=np.float32)
    xc = np.maximum(x, np.float32(-125.0))
    shift = np.float32(12582912.0)
    t = (xc + shift).astype(np.float32)
    j = (t - shift).astype(np.float32)
    f = (xc.astype(np.float64) - j.astype(np.float64)).astype(np.float32)  # exact
    p = (np.float64(c3) * f + np.float64(c2)).astype(np.float32)
    p = (p.astype(np.float64) * f + np.float64(c1)).astype(np.float32)
    p = (p.astype(np.float64) * f + np.float64(c0)).astype(np.float32)
    bits = (p.view(np.uint32).astype(np.uint64) + ((t.view(np.uint32).astype(np.uint64) << 23) & 0xFFFFFFFF))
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32), f


def test_relative_error_over_the_softmax_range():
    x = np.concatenate([
        np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
        np.float32([0.0, 0.5, -0.5, 8.0, -1e-30, 1e-30]),
    ])
    y, f = _exp2_poly(x)
    assert np.all(np.abs(f) <= 0.5)
    rel = np.abs(y.astype(np.float64) / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 7.6e-5, rel.max()  # minimax fit: 7.48e-5; half a bf16 ulp is 2^-9


def test_masked_keys_and_underflow():
    y, _ = _exp2_poly(np.float32([-np.inf, -1e30, -126.0, -200.0]))
    assert np.all(y == y[0]) and abs(float(y[0]) / 2.0 ** -125 - 1.0) < 7.6e-5  # p(0) * 2^-125
    # Next to the row maximum (2^0 = 1) such a term vanishes in an fp32 row sum and in bf16/fp16 P
    # relative to any visible key.
    assert np.float32(1.0) + y[0] == np.float32(1.0)
