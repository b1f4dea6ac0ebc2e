"""tcx_sm100_reduce_all_noalloc: the full-tensor reduction for callers that cannot
allocate device memory (hosts that own the whole device memory budget, or loops
that cannot pay cudaMalloc's device-wide synchronization).

It must return what the regular entry point (tcx_sm100_reduce_all, which takes a
caller workspace) returns, on two calls in a row: the second call reuses the fixed
scratch array the first call left behind. This file is collected last on purpose, so
a run that stops at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from tensorcx_b200 import _abi

pytestmark = pytest.mark.gpu


def _call_regular(lib, op, dtype, x, out):
    ws_bytes = lib.tcx_sm100_reduce_workspace_bytes(x.numel())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _abi.check(lib.tcx_sm100_reduce_all(None, _abi.OP[op], dtype, ctypes.c_void_p(x.data_ptr()), x.numel(),
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws_bytes))
    torch.cuda.synchronize()


def _call_noalloc(lib, op, dtype, x, out):
    _abi.check(lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP[op], dtype, ctypes.c_void_p(x.data_ptr()),
                                                x.numel(), ctypes.c_void_p(out.data_ptr())))
    torch.cuda.synchronize()


@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "argmax"])
@pytest.mark.parametrize("dtype", ["float32", "int32"])
def test_noalloc_matches_regular_entry_point(tcx, op, dtype):
    if op == "mean" and dtype == "int32":
        pytest.skip("mean is float32 only")
    lib = _abi.lib()
    code = _abi.FLOAT32 if dtype == "float32" else _abi.INT32
    rng = np.random.default_rng(17)
    for n in ((1 << 22) + 3, 70000):  # two calls in a row, different sizes and data
        if dtype == "float32":
            host = rng.standard_normal(n, dtype=np.float32)
        else:
            host = rng.integers(-1000, 1000, n).astype(np.int32)
        host[n // 3] = host.max()  # a tie for the index-carrying ops
        x = torch.from_numpy(host).cuda()
        out_dtype = torch.int32 if op == "argmax" else x.dtype
        want = torch.empty((), dtype=out_dtype, device="cuda")
        got = torch.full((), 7, dtype=out_dtype, device="cuda")
        _call_regular(lib, op, code, x, want)
        _call_noalloc(lib, op, code, x, got)
        # same kernels, same fixed reduction order: identical results
        if out_dtype == torch.float32:
            w, g = float(want.item()), float(got.item())
            assert np.float32(w).view(np.uint32) == np.float32(g).view(np.uint32), (op, n, w, g)
        else:
            assert int(want.item()) == int(got.item()), (op, n)


def test_noalloc_rejects_bad_arguments(tcx):
    lib = _abi.lib()
    x = torch.zeros(4, device="cuda")
    out = torch.empty((), device="cuda")
    assert lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["max"], _abi.FLOAT32, ctypes.c_void_p(x.data_ptr()), 0,
                                            ctypes.c_void_p(out.data_ptr())) == _abi.INVALID_ARGUMENT
    assert lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["mean"], _abi.INT32, ctypes.c_void_p(x.data_ptr()), 4,
                                            ctypes.c_void_p(out.data_ptr())) == _abi.INVALID_ARGUMENT
    assert lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["sum"], _abi.FLOAT32, ctypes.c_void_p(x.data_ptr()), -1,
                                            ctypes.c_void_p(out.data_ptr())) == _abi.INVALID_ARGUMENT
