"""Shared pytest configuration: the `gpu` marker and common fixtures.

`-m "not gpu"` runs the CPU suite (oracle vs reference vs golden vectors,
host logic, C-ABI exports); `-m gpu` runs the parity tests on a B200 through
the C ABI of libcormorant_cuda.so.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "big: full-size case, run on the tensor-core path only")


@pytest.fixture(scope="session")
def port():
    import oracle
    p = oracle.port()
    p.set_threads(min(os.cpu_count() or 1, 64))
    return p


@pytest.fixture(scope="session")
def cm():
    """The product library, initialised on cuda:0 (GPU tests only)."""
    import cormorant_b200 as cmb
    cmb.init("0")
    return cmb


@pytest.fixture(params=["tensor", "direct"])
def mac_path(request, cm):
    """Run a MatMul / Conv test on both GPU paths: the split + tcgen05 pipeline (direct
    limit 0) and the one-kernel CUDA-core path for launch-bound sizes (limit 2^26 MACs)."""
    from cormorant_b200 import _lib
    if request.param == "direct" and request.node.get_closest_marker("big"):
        pytest.skip("full-size case: above the direct-path limit")
    L = _lib.lib()
    old = L.cm_set_direct_limit(0 if request.param == "tensor" else (1 << 26))
    yield request.param
    L.cm_set_direct_limit(old)
