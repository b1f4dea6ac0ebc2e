"""tensorcx_b200 — B200 (sm_100a) CUDA backend for tensor.cx's data-parallel hot path.

The product is libtcx_sm100.so behind the C ABI in include/tcx_sm100.h. This package
holds its sources (csrc/), the in-tree build (build.py), the ctypes binding (_abi.py),
the host-side shape planning (plan.py) and a Python mirror of the tensor.cx op API on
CUDA tensors (ops.py).
"""
from ._abi import lib  # noqa: F401
from . import plan  # noqa: F401

__all__ = ["lib", "plan", "ops"]


def __getattr__(name):
    if name == "ops":
        import importlib
        return importlib.import_module(".ops", __name__)
    raise AttributeError(name)
