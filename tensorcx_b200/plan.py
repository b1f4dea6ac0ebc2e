"""Host-side shape planning of the tensor.cx core, as the sm_100a backend consumes it.

Same plans, argument meaning and error behaviour as cpp/tensorcx/core/shape.cpp
(make_matmul_plan 49-76, make_reduction_plan 140-172, make_broadcast_plan 202-229)
and the axis normalisation of cpu_backend.cpp:76-123; errors are ValueError, as the
bindings report kInvalidArgument. The C++ host backend uses the core's own plans;
this module serves the Python host mirror (tensorcx_b200.ops).
"""
from __future__ import annotations

from dataclasses import dataclass

_MAX = (1 << 63) - 1


def _mul(a: int, b: int, what: str) -> int:
    if a and b > _MAX // a:
        raise ValueError(what)
    return a * b


def numel(shape) -> int:
    total = 1
    for d in shape:
        if d < 0:
            raise ValueError("shape dimensions must be non-negative")
        total = _mul(total, d, "shape size overflow")
    return total


def strides(shape) -> list[int]:
    out, s = [0] * len(shape), 1
    for i in reversed(range(len(shape))):
        if shape[i] < 0:
            raise ValueError("shape dimensions must be non-negative")
        out[i] = s
        s = _mul(s, shape[i], "shape stride overflow")
    return out


@dataclass
class MatmulPlan:
    output_shape: list
    batch_shape: list
    lhs_batch_strides: list
    rhs_batch_strides: list
    m: int
    k: int
    n: int


def matmul(lhs, rhs) -> MatmulPlan:
    lhs, rhs = list(lhs), list(rhs)
    if not lhs or not rhs:
        raise ValueError("matmul requires rank >= 1 tensors")
    numel(lhs), numel(rhs)
    ls, rs = strides(lhs), strides(rhs)
    lvec, rvec = len(lhs) == 1, len(rhs) == 1
    m, k = (1 if lvec else lhs[-2]), lhs[-1]
    rk, n = (rhs[0] if rvec else rhs[-2]), (1 if rvec else rhs[-1])
    if k != rk:
        raise ValueError("matmul shape mismatch: contracting dimensions differ")
    lb, rb = (0 if lvec else len(lhs) - 2), (0 if rvec else len(rhs) - 2)
    rank = max(lb, rb)
    shape, lst, rst = [1] * rank, [0] * rank, [0] * rank
    for a in range(rank):
        li, ri = a - (rank - lb), a - (rank - rb)
        l = lhs[li] if li >= 0 else 1
        r = rhs[ri] if ri >= 0 else 1
        if l != r and 1 not in (l, r):
            raise ValueError("matmul batch dimensions cannot broadcast")
        shape[a] = r if l == 1 else l
        if li >= 0 and l != 1:
            lst[a] = ls[li]
        if ri >= 0 and r != 1:
            rst[a] = rs[ri]
    out = shape + ([] if lvec else [m]) + ([] if rvec else [n])
    numel(out), strides(out)
    return MatmulPlan(out, shape, lst, rst, m, k, n)


def broadcast(lhs, rhs):
    """(output shape, lhs strides, rhs strides) with zero strides on broadcast axes."""
    lhs, rhs = list(lhs), list(rhs)
    numel(lhs), numel(rhs)
    lc, rc = strides(lhs), strides(rhs)
    rank = max(len(lhs), len(rhs))
    lp, rp = rank - len(lhs), rank - len(rhs)
    out, lst, rst = [], [], []
    for a in range(rank):
        l = lhs[a - lp] if a >= lp else 1
        r = rhs[a - rp] if a >= rp else 1
        if l != r and 1 not in (l, r):
            raise ValueError("shape mismatch: tensor shapes are not broadcastable")
        out.append(r if l == 1 else l)
        lst.append(lc[a - lp] if a >= lp and l != 1 else 0)
        rst.append(rc[a - rp] if a >= rp and r != 1 else 0)
    numel(out), strides(out)
    return out, lst, rst


@dataclass
class ReductionPlan:
    output_shape: list
    index_metadata: list  # (extent, stride) pairs: kept axes, then reduced axes
    reduction_size: int


def reduction(shape, axes) -> ReductionPlan:
    shape = list(shape)
    numel(shape)
    st = strides(shape)
    rank = len(shape)
    chosen = set()
    for a in axes:
        a = a + rank if a < 0 else a
        if not 0 <= a < rank:
            raise ValueError("reduction axis is out of range")
        if a in chosen:
            raise ValueError("reduction axes must not repeat")
        chosen.add(a)
    kept = [a for a in range(rank) if a not in chosen]
    red = [a for a in range(rank) if a in chosen]
    meta = []
    for a in kept + red:
        meta += [shape[a], st[a]]
    out = [shape[a] for a in kept]
    count = numel(out)
    strides(out)
    if any(shape[a] == 0 for a in red):
        size = 0
    elif count:
        size = numel([shape[a] for a in red])
    else:
        size = 1  # unvisited sentinel, as the core does
    return ReductionPlan(out, meta, size)


def axis(shape, ax: int):
    """(output shape, outer, reduce, inner) of a one-axis primitive."""
    shape = list(shape)
    rank = len(shape)
    if rank == 0:
        if ax in (0, -1):
            return [], 1, 1, 1
        raise ValueError("reduction axis is out of range")
    a = ax + rank if ax < 0 else ax
    if not 0 <= a < rank:
        raise ValueError("reduction axis is out of range")
    return shape[:a] + shape[a + 1:], numel(shape[:a]), shape[a], strides(shape)[a]


def epsilon(eps: float) -> float:
    import math
    import struct
    if not math.isfinite(eps) or eps < 0 or eps > 3.4028234663852886e38:
        raise ValueError("epsilon must be finite and non-negative and representable as float32")
    f = struct.unpack("f", struct.pack("f", eps))[0]
    if eps > 0 and f == 0.0:
        raise ValueError("epsilon must be finite and non-negative and representable as float32")
    return f
