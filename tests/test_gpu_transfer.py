"""Synchronous host <-> device copies of the C ABI (tcx_sm100_copy_to_device / _host):
pageable buffers staged through the pinned two-slot ring with parallel host copies,
page-locked buffers and small copies direct. Every byte must arrive unchanged."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MIB = 1 << 20


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("nbytes", [0, 1, 4095, 4 * MIB - 4, 4 * MIB, 4 * MIB + 12, 32 * MIB, 70 * MIB + 4,
                                    200 * MIB + 8])
def test_pageable_round_trip(tcx, nbytes):
    from tensorcx_b200._abi import check, lib
    src = np.random.default_rng(nbytes).integers(0, 256, nbytes, dtype=np.uint8)
    dev = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    check(lib().tcx_sm100_copy_to_device(stream(), ctypes.c_void_p(dev.data_ptr()),
                                         src.ctypes.data_as(ctypes.c_void_p), nbytes))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev[:nbytes].cpu().numpy(), src)
    dev[:nbytes].add_(1)  # change it on the device, then bring it back
    back = np.empty(nbytes, np.uint8)
    check(lib().tcx_sm100_copy_to_host(stream(), back.ctypes.data_as(ctypes.c_void_p),
                                       ctypes.c_void_p(dev.data_ptr()), nbytes))
    np.testing.assert_array_equal(back, (src + 1).astype(np.uint8))


def test_page_locked_and_unaligned(tcx):
    from tensorcx_b200._abi import check, lib
    n = 9 * MIB + 3
    pinned = torch.randint(0, 256, (n + 5,), dtype=torch.uint8).pin_memory()
    dev = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(lib().tcx_sm100_copy_to_device(stream(), ctypes.c_void_p(dev.data_ptr()),
                                         ctypes.c_void_p(pinned.data_ptr() + 5), n))
    assert torch.equal(dev.cpu(), pinned[5:])
    odd = np.zeros(n + 3, np.uint8)  # pageable destination at an odd address
    check(lib().tcx_sm100_copy_to_host(stream(), ctypes.c_void_p(odd.ctypes.data + 3),
                                       ctypes.c_void_p(dev.data_ptr()), n))
    np.testing.assert_array_equal(odd[3:], pinned[5:].numpy())


def test_missing_buffer_is_invalid(tcx):
    from tensorcx_b200._abi import check, lib
    with pytest.raises(ValueError):
        check(lib().tcx_sm100_copy_to_device(stream(), None, None, 16))
