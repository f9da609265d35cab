"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs on any machine (oracle vs golden vectors, host logic, C-ABI symbol
checks, gloo multi-process tests); `-m gpu` needs a B200 and runs the parity tests through
the C ABI.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flash-attn-from-scratch_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; parity tests through the C ABI")


import pytest


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: no kernel may have recorded a device-side failure."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import llm_kernels

    code, site, blk, thr = llm_kernels.device_status()
    if code:
        llm_kernels.clear_device_status()
        pytest.fail(f"device status {code} at site {site} (block {blk}, thread {thr})")
