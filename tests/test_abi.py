"""The C-ABI library loads, exports every symbol include/*.h declares, and rejects
malformed arguments on the host before touching the GPU (no device needed)."""
import ctypes
import glob
import os
import re

import pytest

from tensorcx_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(tcx_sm100_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    assert len(declared_symbols()) >= 19


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports(name):
    lib = _abi.lib()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert name in _abi.SIGNATURES, f"{name} has no ctypes signature"


def test_no_cpu_fallback_symbols():
    """The product library links no oracle or reference code."""
    out = os.popen(f"nm -D {_abi.LIB_PATH}").read()
    assert "tcxo_" not in out and "tcxref_" not in out and "CpuBackend" not in out


def test_abi_version_and_errors():
    lib = _abi.lib()
    assert lib.tcx_sm100_abi_version() >= 1
    # invalid arguments are rejected before any CUDA call, with a message
    rc = lib.tcx_sm100_matmul(None, None, None, None, -1, 2, 2, 1, None, None, None, 0, None, 0, 0, None, 0)
    assert rc == _abi.INVALID_ARGUMENT
    assert b"negative" in lib.tcx_sm100_last_error()
    rc = lib.tcx_sm100_axis(None, 99, 0, None, None, 1, 1, 1, 0.0, None, 0)
    assert rc == _abi.INVALID_ARGUMENT
    rc = lib.tcx_sm100_binary(None, _abi.OP["divide"], _abi.INT32, None, None, None, 4, None, 0)
    assert rc == _abi.INVALID_ARGUMENT and b"float32" in lib.tcx_sm100_last_error()
    rc = lib.tcx_sm100_min_argmax(None, _abi.OP["min"], 0, None, None, 1, 0, None, 0, None, 0)
    assert rc == _abi.INVALID_ARGUMENT
    rc = lib.tcx_sm100_reduce_all(None, _abi.OP["max"], 0, None, 0, None, None, 0)
    assert rc == _abi.INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _abi.check(_abi.INVALID_ARGUMENT)


def test_more_entry_points_reject_bad_arguments_before_cuda():
    """Unsupported ops, negative or empty extents and missing buffers come back as
    TCX_INVALID_ARGUMENT with a message, before any CUDA call (this runs without a GPU)."""
    lib = _abi.lib()
    cases = [
        # no-allocation full reduction: op / dtype checked first, then the count
        (lambda: lib.tcx_sm100_reduce_all_noalloc(None, 99, 0, None, 4, None), b"op"),
        (lambda: lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["sum"], 0, None, -1, None), b"negative"),
        (lambda: lib.tcx_sm100_reduce_partial(None, _abi.OP["sum"], 0, None, 0, 0, None, None, 0), b"non-empty"),
        (lambda: lib.tcx_sm100_affine_norm(None, _abi.OP["layernorm"], None, None, -1, 4, 1, 1e-5, None, None),
         b"negative"),
        (lambda: lib.tcx_sm100_affine_norm(None, _abi.OP["softmax"], None, None, 1, 4, 1, 1e-5, None, None),
         b"rmsnorm"),
        (lambda: lib.tcx_sm100_copy_to_device(None, None, None, 16), b"buffer"),
    ]
    for call, word in cases:
        assert call() == _abi.INVALID_ARGUMENT
        assert word in lib.tcx_sm100_last_error(), lib.tcx_sm100_last_error()


def test_workspace_queries():
    lib = _abi.lib()
    assert lib.tcx_sm100_matmul_workspace_bytes(8192, 8192, 8192, 1, 1, 0) >= 4 * 4 * 8192 * 8192
    assert lib.tcx_sm100_matmul_workspace_bytes(32, 64, 128, 1, 1, 0) == 0  # FFMA: no scratch
    assert lib.tcx_sm100_axis_workspace_bytes(_abi.OP["softmax"], 4, 1 << 20, 1) == 0
