"""The division-free int8 codes used for fp16 / bf16 values are the IEEE-division codes for
every input the format can hold (CPU, exhaustive: ~1e9 (x, absmax) pairs per format).

The quantiser's fp16 / bf16 path and the int8 GEMM's re-quantising epilogue compute
rint(x / scale) as rint of Markstein's FMA-corrected reciprocal product instead of dividing;
``exhaustive_codes.c`` enumerates every pair (x, absmax) with |x| <= absmax and compares.
The GPU tests then check the kernels themselves against the oracle.
"""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path_factory.mktemp("exh") / "exhaustive_codes")
    flags = ["-O2", "-ffp-contract=off"]
    # Hardware FMA when the host has it (fmaf is correctly rounded either way).
    r = subprocess.run([cc, *flags, "-mfma", "-o", exe, os.path.join(HERE, "exhaustive_codes.c"), "-lm"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        r = subprocess.run([cc, *flags, "-o", exe, os.path.join(HERE, "exhaustive_codes.c"), "-lm"],
                           capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


@pytest.mark.parametrize("fmt", ["f", "b"])
def test_fma_corrected_codes_equal_division_codes(checker, fmt):
    r = subprocess.run([checker, fmt], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    fields = dict(kv.split("=") for kv in r.stdout.split()[1:])
    assert int(fields["mismatches"]) == 0
    assert int(fields["pairs"]) > 10 ** 9
