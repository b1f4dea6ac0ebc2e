"""Test configuration: the `gpu` marker, repo import path and shared fixtures.

`-m "not gpu"` runs on any machine (oracle pins, C-ABI symbol checks, host logic,
multi-process gloo tests). `-m gpu` runs the parity tests through the C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); runs the CUDA kernels")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref/libtcx_ref.so not built (reference sources absent)")
    return Reference()


@pytest.fixture(scope="session")
def tcx():
    """The product's op mirror on cuda:0; fails (not skips) when the GPU or the
    library is missing, so a GPU run can never pass on a fallback."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.set_device(0)
    from tensorcx_b200 import _abi, ops
    assert _abi.lib().tcx_sm100_device_supported(0) == 0, _abi.lib().tcx_sm100_last_error()
    return ops
