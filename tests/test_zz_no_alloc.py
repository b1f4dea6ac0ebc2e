"""tcx_sm100_reduce_all_noalloc: the full-tensor reduction for callers that cannot
allocate device memory (hosts that own the whole device memory budget, or loops
that cannot pay cudaMalloc's device-wide synchronization).

It must return what the regular entry point (tcx_sm100_reduce_all, which takes a
caller workspace) returns, on two calls in a row: the second call reuses the fixed
scratch array the first call left behind. Each result is also checked against the
CPU oracle on its own (bit-exact for int32, max, min and argmax; float32 sum and
mean within 1e-5 relative of the CPU, or closer to the float64 sum than the CPU's
own result), so a fault the two entry points shared would still show. This file is
collected last on purpose, so a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from tensorcx_b200 import _abi

pytestmark = pytest.mark.gpu

CASES = [(op, dt) for dt in ("float32", "int32") for op in ("sum", "mean", "max", "min", "argmax")
         if not (op == "mean" and dt == "int32")]  # mean is float32 only (rejected below)


def _call_regular(lib, op, dtype, x, out):
    ws_bytes = lib.tcx_sm100_reduce_workspace_bytes(x.numel())
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    _abi.check(lib.tcx_sm100_reduce_all(None, _abi.OP[op], dtype, ctypes.c_void_p(x.data_ptr()), x.numel(),
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws_bytes))
    torch.cuda.synchronize()


def _call_noalloc(lib, op, dtype, x, out):
    _abi.check(lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP[op], dtype, ctypes.c_void_p(x.data_ptr()),
                                                x.numel(), ctypes.c_void_p(out.data_ptr())))
    torch.cuda.synchronize()


def _oracle_value(oracle, op, host):
    return np.asarray(getattr(oracle, op)(host)).reshape(())


def _check_against_oracle(oracle, op, host, got):
    want = _oracle_value(oracle, op, host)
    if op in ("sum", "mean") and host.dtype == np.float32:
        exact = oracle.sum_f64(host) / (host.size if op == "mean" else 1)
        g, w = float(got), float(want)
        assert abs(g - w) <= 1e-5 * abs(w) or abs(g - exact) <= abs(w - exact), (op, g, w, exact)
    elif host.dtype == np.float32 and op != "argmax":
        assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (op, got, want)
    else:
        assert int(got) == int(want), (op, got, want)


@pytest.mark.parametrize("op,dtype", CASES)
def test_noalloc_matches_regular_entry_point(tcx, oracle, op, dtype):
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
        _check_against_oracle(oracle, op, host, got.item())


@pytest.mark.parametrize("dtype", ["float32", "int32"])
def test_noalloc_empty_input(tcx, dtype):
    """An empty sum is 0 and an empty mean is NaN (0/0), as in the reference's CPU
    reduction; the output is overwritten, not left as it was."""
    lib = _abi.lib()
    code = _abi.FLOAT32 if dtype == "float32" else _abi.INT32
    tdt = torch.float32 if dtype == "float32" else torch.int32
    x = torch.zeros(4, dtype=tdt, device="cuda")
    out = torch.full((), 5, dtype=tdt, device="cuda")
    _abi.check(lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["sum"], code, ctypes.c_void_p(x.data_ptr()), 0,
                                                ctypes.c_void_p(out.data_ptr())))
    torch.cuda.synchronize()
    assert out.item() == 0
    if dtype == "float32":
        out.fill_(5)
        _abi.check(lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["mean"], code, ctypes.c_void_p(x.data_ptr()), 0,
                                                    ctypes.c_void_p(out.data_ptr())))
        torch.cuda.synchronize()
        assert np.isnan(out.item())


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


def test_noalloc_on_every_visible_device(oracle):
    """The scratch address is looked up per device; each GPU gets its own."""
    n_dev = torch.cuda.device_count()
    if n_dev < 2:
        pytest.skip("one GPU visible: the per-device set-up is covered by the tests above")
    lib = _abi.lib()
    rng = np.random.default_rng(5)
    host = rng.integers(-1000, 1000, 100000).astype(np.int32)
    for dev in range(n_dev):
        with torch.cuda.device(dev):
            x = torch.from_numpy(host).to(f"cuda:{dev}")
            out = torch.full((), 7, dtype=torch.int32, device=f"cuda:{dev}")
            _abi.check(lib.tcx_sm100_reduce_all_noalloc(None, _abi.OP["sum"], _abi.INT32,
                                                        ctypes.c_void_p(x.data_ptr()), x.numel(),
                                                        ctypes.c_void_p(out.data_ptr())))
            torch.cuda.synchronize()
            assert int(out.item()) == int(oracle.sum(host))
