"""ctypes binding of include/tcx_sm100.h (the C ABI of libtcx_sm100.so).

This is the binding a tensor.cx maintainer would write for the C ABI from Python;
the C++ host backend calls the same symbols directly. Loading fails loudly when the
library is not built: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libtcx_sm100.so")

OK, INVALID_ARGUMENT, UNAVAILABLE, INTERNAL = 0, 1, 2, 3
FLOAT32, INT32, BOOL = 0, 1, 2
OP = dict(add=1, multiply=2, matmul=3, sum=4, max=5, mean=6, exp=7, gelu=8, silu=9, softmax=10,
          rmsnorm=11, layernorm=12, subtract=13, divide=14, negate=15, add_scalar=16, subtract_scalar=17,
          multiply_scalar=18, divide_scalar=19, equal=24, not_equal=25, less=26, less_equal=27, greater=28,
          greater_equal=29, logical_and=30, logical_or=31, logical_xor=32, logical_not=33, where=34, any=35,
          all=36, log=38, sqrt=39, abs=40, min=41, argmax=42, clip=43, topk=44)
ACT = dict(none=0, silu=1, relu=2)
MATMUL_PATH = dict(auto=0, ffma=1, tensor=2)
RANDOM = dict(normal=0, uniform=1)

_vp, _i64, _sz, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_int32, ctypes.c_float
_i64p = ctypes.POINTER(ctypes.c_int64)


class Partial(ctypes.Structure):
    """tcx_partial: one shard's record of a full-tensor reduction (16 bytes)."""
    _fields_ = [("key", ctypes.c_uint32), ("bits", ctypes.c_uint32), ("index", ctypes.c_int64)]


# name -> (restype, argtypes); every symbol include/tcx_sm100.h declares
SIGNATURES = {
    "tcx_sm100_last_error": (ctypes.c_char_p, []),
    "tcx_sm100_abi_version": (ctypes.c_int, []),
    "tcx_sm100_device_supported": (ctypes.c_int, [ctypes.c_int]),
    "tcx_sm100_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "tcx_sm100_timer_enable": (ctypes.c_int, [ctypes.c_int]),
    "tcx_sm100_timer_read": (ctypes.c_int, [ctypes.c_char_p, _sz, _i64p, ctypes.POINTER(ctypes.c_double), _i32,
                                            ctypes.POINTER(ctypes.c_int32)]),
    "tcx_sm100_axis": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64, _i64, _f32, _vp, _sz]),
    "tcx_sm100_axis_workspace_bytes": (_sz, [ctypes.c_int, _i64, _i64, _i64]),
    "tcx_sm100_affine_norm": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp]),
    "tcx_sm100_reduce_axes": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64, _i64p,
                                             _i32, _i32, _vp, _sz]),
    "tcx_sm100_min_argmax": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64, _i64p, _i32,
                                            _vp, _sz]),
    "tcx_sm100_reduce_workspace_bytes": (_sz, [_i64]),
    "tcx_sm100_reduce_all": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _i64, _vp, _vp, _sz]),
    "tcx_sm100_reduce_all_noalloc": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _i64, _vp]),
    "tcx_sm100_reduce_partial": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _i64, _i64, _vp, _vp, _sz]),
    "tcx_sm100_reduce_combine": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _i32, _i64, _vp]),
    "tcx_sm100_mailbox_bytes": (_sz, [_i32]),
    "tcx_sm100_mailbox_create": (ctypes.c_int, [_i32, ctypes.POINTER(_vp), _vp]),
    "tcx_sm100_mailbox_open": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "tcx_sm100_mailbox_close": (ctypes.c_int, [_vp]),
    "tcx_sm100_mailbox_free": (ctypes.c_int, [_vp]),
    "tcx_sm100_reduce_sharded": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _i64, _i64, ctypes.POINTER(_vp),
                                                _i32, _i32, ctypes.c_uint64, ctypes.c_uint64, _i64, _vp, _vp, _sz]),
    "tcx_sm100_unary": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64]),
    "tcx_sm100_binary": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _i64, _i64p, _i32]),
    "tcx_sm100_clip": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64p, _i32]),
    "tcx_sm100_bias_act": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_int]),
    "tcx_sm100_fill": (ctypes.c_int, [_vp, _vp, _i64, ctypes.c_uint32]),
    "tcx_sm100_linear_workspace_bytes": (_sz, [_i64, _i64, _i64, ctypes.c_int]),
    "tcx_sm100_linear": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                        _vp, _sz]),
    "tcx_sm100_matmul_host_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "tcx_sm100_matmul_host": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz]),
    "tcx_sm100_attention_softmax": (ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _i64p, _i64p, _i64p, _i32, _f32,
                                                   _i32]),
    "tcx_sm100_attention_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32]),
    "tcx_sm100_attention": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64p,
                                           _i64p, _i64p, _i64p, _i32, _i64p, _f32, _i32, _vp, _sz]),
    "tcx_sm100_copy_to_device": (ctypes.c_int, [_vp, _vp, _vp, _sz]),
    "tcx_sm100_copy_to_host": (ctypes.c_int, [_vp, _vp, _vp, _sz]),
    "tcx_sm100_random": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _i64, ctypes.c_uint64, ctypes.c_uint64, _f32, _f32]),
    "tcx_sm100_map": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, ctypes.c_double, _i32]),
    "tcx_sm100_cast": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _vp]),
    "tcx_sm100_predicate": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64p, _i32]),
    "tcx_sm100_bool_reduce": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64, _i64, _i64p, _i32]),
    "tcx_sm100_index_copy": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i64, _i64p, _i64p, _i32, _i64]),
    "tcx_sm100_concat": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64]),
    "tcx_sm100_masked_select_workspace_bytes": (_sz, [_i64]),
    "tcx_sm100_masked_select_count": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _sz]),
    "tcx_sm100_masked_select": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i64, _i64, _vp, _vp, _sz]),
    "tcx_sm100_topk": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32]),
    "tcx_sm100_embedding": (ctypes.c_int, [_vp, _vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "tcx_sm100_matmul_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, ctypes.c_int]),
    "tcx_sm100_matmul": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64p, _i64p, _i64p, _i32,
                                        _vp, ctypes.c_int, ctypes.c_int, _vp, _sz]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use; raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m tensorcx_b200.build` "
                "(tensorcx_b200 has no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class TcxError(RuntimeError):
    pass


def check(status: int) -> None:
    """Maps a C-ABI status to the exceptions the tensor.cx bindings raise
    (bindings/python_module.cpp:402-414): invalid argument -> ValueError."""
    if status == OK:
        return
    message = lib().tcx_sm100_last_error().decode()
    if status == INVALID_ARGUMENT:
        raise ValueError(message)
    raise TcxError(message or f"tcx_sm100 status {status}")


def i64_array(values):
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)
