"""TEST INFRASTRUCTURE ONLY — CPU checkers for the tensor.cx hot path.

Two interchangeable checkers with the same method names as the tensor.cx Python API
(python/tensorcx/tensor.py: matmul 500-505, sum/max/mean 508-545, softmax/rmsnorm/
layernorm 565-584, min/argmax 834-855, clip 858-876):

* ``Oracle``    — the plain-C restatement in tcx_oracle.c, with the shape planning of
                  cpp/tensorcx/core/shape.cpp restated here in Python.
* ``Reference`` — the reference's own CPU backend, compiled from its sources into
                  _ref/libtcx_ref.so (absent when the reference tree was not there at
                  build time; ``Reference.available()`` says so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module, and only
as the checker or the timed CPU baseline. The product never imports it.
Invalid arguments raise ValueError, as the reference bindings map kInvalidArgument
(bindings/python_module.cpp:402-414).
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libtcx_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtcx_ref.so")

# tensorcx::OpKind values (cpp/tensorcx/core/operation.h:12-63)
OPKIND = {name: i for i, name in enumerate([
    "fill", "add", "multiply", "matmul", "sum", "max", "mean", "exp", "gelu", "silu",
    "softmax", "rmsnorm", "layernorm", "subtract", "divide", "negate", "add_scalar",
    "subtract_scalar", "multiply_scalar", "divide_scalar", "cast", "transpose", "slice",
    "concat", "equal", "not_equal", "less", "less_equal", "greater", "greater_equal",
    "logical_and", "logical_or", "logical_xor", "logical_not", "where", "any", "all",
    "masked_select", "log", "sqrt", "abs", "min", "argmax", "clip", "topk", "linear",
    "affine_rmsnorm", "affine_layernorm", "embedding", "attention", "attention_softmax"])}

_I64P = ctypes.POINTER(ctypes.c_int64)


def _i64(values: Sequence[int]):
    arr = (ctypes.c_int64 * max(1, len(values)))(*values)
    return arr


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return 0
    if a.dtype == np.int32:
        return 1
    raise ValueError("only float32 and int32 tensors are on this path")


# ---------------------------------------------------------------- shape planning
# Restated from cpp/tensorcx/core/shape.cpp (numel 25-36, contiguous_strides 38-47,
# make_matmul_plan 49-76, matmul_batch_offset 78-85, make_reduction_plan 140-172,
# make_broadcast_plan 202-229). Overflow checks raise ValueError like the reference's
# std::invalid_argument.
_DIM_MAX = 2**63 - 1


def numel(shape) -> int:
    total = 1
    for d in shape:
        if d < 0:
            raise ValueError("shape dimensions must be non-negative")
        if total != 0 and d > _DIM_MAX // total:
            raise ValueError("shape size overflow")
        total *= d
    return total


def contiguous_strides(shape):
    strides = [1] * len(shape)
    stride = 1
    for i in range(len(shape) - 1, -1, -1):
        if shape[i] < 0:
            raise ValueError("shape dimensions must be non-negative")
        strides[i] = stride
        if stride != 0 and shape[i] > _DIM_MAX // stride:
            raise ValueError("shape stride overflow")
        stride *= shape[i]
    return strides


def matmul_plan(lhs, rhs):
    if not lhs or not rhs:
        raise ValueError("matmul requires rank >= 1 tensors")
    numel(lhs), numel(rhs)
    ls, rs = contiguous_strides(lhs), contiguous_strides(rhs)
    lv, rv = len(lhs) == 1, len(rhs) == 1
    m = 1 if lv else lhs[-2]
    k = lhs[-1]
    rk = rhs[0] if rv else rhs[-2]
    n = 1 if rv else rhs[-1]
    if k != rk:
        raise ValueError("matmul shape mismatch: contracting dimensions differ")
    lb = 0 if lv else len(lhs) - 2
    rb = 0 if rv else len(rhs) - 2
    rank = max(lb, rb)
    batch, lst, rst = [1] * rank, [0] * rank, [0] * rank
    for axis in range(rank):
        has_l, has_r = axis >= rank - lb, axis >= rank - rb
        li, ri = axis - (rank - lb), axis - (rank - rb)
        l = lhs[li] if has_l else 1
        r = rhs[ri] if has_r else 1
        if l != r and l != 1 and r != 1:
            raise ValueError("matmul batch dimensions cannot broadcast")
        batch[axis] = r if l == 1 else l
        if has_l and l != 1:
            lst[axis] = ls[li]
        if has_r and r != 1:
            rst[axis] = rs[ri]
    out = list(batch)
    if not lv:
        out.append(m)
    if not rv:
        out.append(n)
    numel(out), contiguous_strides(out)
    return out, batch, lst, rst, m, k, n


def batch_offset(batch, shape, strides):
    off = 0
    for axis in range(len(shape) - 1, -1, -1):
        off += (batch % shape[axis]) * strides[axis]
        batch //= shape[axis]
    return off


def reduction_plan(shape, axes):
    numel(shape)
    strides = contiguous_strides(shape)
    rank = len(shape)
    selected = [False] * rank
    for axis in axes:
        if axis < 0:
            axis += rank
        if axis < 0 or axis >= rank:
            raise ValueError("reduction axis is out of range")
        if selected[axis]:
            raise ValueError("reduction axes must not repeat")
        selected[axis] = True
    out, meta, reduced = [], [], []
    for a in range(rank):
        if selected[a]:
            reduced.append(shape[a])
        else:
            out.append(shape[a])
            meta += [shape[a], strides[a]]
    for a in range(rank):
        if selected[a]:
            meta += [shape[a], strides[a]]
    count = numel(out)
    contiguous_strides(out)
    if 0 in reduced:
        size = 0
    elif count != 0:
        size = numel(reduced)
    else:
        size = 1
    return out, meta, size


def broadcast_plan(lhs, rhs):
    numel(lhs), numel(rhs)
    lc, rc = contiguous_strides(lhs), contiguous_strides(rhs)
    rank = max(len(lhs), len(rhs))
    out, ls, rs = [0] * rank, [0] * rank, [0] * rank
    lp, rp = rank - len(lhs), rank - len(rhs)
    for axis in range(rank):
        left = 1 if axis < lp else lhs[axis - lp]
        right = 1 if axis < rp else rhs[axis - rp]
        if left != right and left != 1 and right != 1:
            raise ValueError("shape mismatch: tensor shapes are not broadcastable")
        out[axis] = right if left == 1 else left
        if axis >= lp and left != 1:
            ls[axis] = lc[axis - lp]
        if axis >= rp and right != 1:
            rs[axis] = rc[axis - rp]
    numel(out), contiguous_strides(out)
    return out, ls, rs


def checked_scale(scale: float) -> float:
    """checked_scale, core/inference.cpp:15-20: finite, representable as float32, and
    not flushed to zero."""
    narrowed = float(np.float32(scale)) if math.isfinite(scale) and abs(scale) <= 3.4028234663852886e38 else math.inf
    if not math.isfinite(scale) or not math.isfinite(narrowed) or (scale != 0 and narrowed == 0):
        raise ValueError("attention scale must be finite and representable as float32")
    return narrowed


def attention_batch(qs, ks, vs):
    """The batch shape and feature count of the attention composite
    (core/inference.cpp:128-148)."""
    for s in (qs, ks, vs):
        if len(s) < 2:
            raise ValueError("attention tensors require rank >= 2")
    features = qs[-1]
    if features <= 0 or features != ks[-1] or ks[-2] != vs[-2]:
        raise ValueError("attention query/key features and key/value sequence sizes must match; "
                         "features must be positive")
    batch = []
    for s in (qs, ks, vs):
        inp = list(s[:-2])
        rank = max(len(batch), len(inp))
        merged = []
        for a in range(rank):
            left = 1 if a < rank - len(batch) else batch[a - (rank - len(batch))]
            right = 1 if a < rank - len(inp) else inp[a - (rank - len(inp))]
            if left != right and left != 1 and right != 1:
                raise ValueError("attention batch dimensions cannot broadcast")
            merged.append(right if left == 1 else left)
        batch = merged
    return batch, features


def axis_dims(shape, axis):
    """reduction_dims of cpu_backend.cpp:76-123: (output shape, outer, reduce, inner)."""
    rank = len(shape)
    if rank == 0:
        if axis in (0, -1):
            return [], 1, 1, 1
        raise ValueError("reduction axis is out of range")
    if axis < 0:
        axis += rank
    if axis < 0 or axis >= rank:
        raise ValueError("reduction axis is out of range")
    out = [d for i, d in enumerate(shape) if i != axis]
    outer = numel(shape[:axis])
    inner = contiguous_strides(shape)[axis]
    return out, outer, shape[axis], inner


def checked_epsilon(eps: float) -> float:
    """cpu_backend.cpp:30-42."""
    if not math.isfinite(eps) or eps < 0 or eps > float(np.finfo(np.float32).max):
        raise ValueError("epsilon must be finite and non-negative and representable as float32")
    rounded = float(np.float32(eps))
    if eps > 0 and rounded == 0.0:
        raise ValueError("epsilon must be finite and non-negative and representable as float32")
    return rounded


def axes_for(shape, axis):
    """Dispatch of python/tensorcx/tensor.py:_reduce (508-529): returns
    ('axis', a) for the original single-axis primitive or ('axes', tuple)."""
    rank = len(shape)
    if axis is None:
        axes = tuple(range(rank))
        scalar = rank == 0
    else:
        values = tuple(axis) if isinstance(axis, (tuple, list)) else (axis,)
        scalar = rank == 0 and len(values) == 1 and values[0] in (0, -1)
        if scalar:
            axes = ()
        else:
            axes = []
            for v in values:
                if v < -rank or v >= rank:
                    raise ValueError("reduction axis is out of range")
                axes.append(v % rank if rank else v)
            axes = tuple(axes)
    if scalar or len(axes) == 1:
        return "axis", (axes[0] if axes else 0)
    return "axes", axes


class _Lib:
    def __init__(self, path):
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built (run `make -C oracle`)")
        self.lib = ctypes.CDLL(path)


class Oracle(_Lib):
    """The C restatement (tcx_oracle.c) behind the tensor.cx op names."""

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path)
        L = self.lib
        L.tcxo_sum_f64.restype = ctypes.c_double

    # --------------------------------------------------------------- reductions
    def _reduce(self, name, x, axis):
        op = {"sum": 0, "max": 1, "mean": 2}[name]
        x = np.ascontiguousarray(x)
        dt = _dtype_code(x)
        if name == "mean" and dt != 0:
            raise ValueError("mean only supports float32 tensors")
        mode, sel = axes_for(list(x.shape), axis)
        if mode == "axis":
            out_shape, outer, reduce, inner = axis_dims(list(x.shape), sel)
            if name == "max" and reduce == 0:
                raise ValueError("max reduction requires a non-empty axis")
            out = np.empty(out_shape, dtype=x.dtype)
            fn = self.lib.tcxo_reduce_axis_f32 if dt == 0 else self.lib.tcxo_reduce_axis_i32
            fn(op, _ptr(x), _ptr(out), ctypes.c_int64(outer), ctypes.c_int64(reduce),
               ctypes.c_int64(inner))
            return out
        out_shape, meta, size = reduction_plan(list(x.shape), sel)
        if name == "max" and size == 0:
            raise ValueError("max reduction requires non-empty axes")
        if not sel:
            return x.copy()
        out = np.empty(out_shape, dtype=x.dtype)
        groups = numel(out_shape)
        if groups:
            self.lib.tcxo_reduce_axes(op, dt, _ptr(x), _ptr(out), ctypes.c_int64(groups),
                                      ctypes.c_int64(size), _i64(meta),
                                      ctypes.c_int64(len(out_shape)), ctypes.c_int64(x.ndim))
        return out

    def sum(self, x, axis=None):
        return self._reduce("sum", x, axis)

    def max(self, x, axis=None):
        return self._reduce("max", x, axis)

    def mean(self, x, axis=None):
        return self._reduce("mean", x, axis)

    def _min_argmax(self, code, x, axis):
        x = np.ascontiguousarray(x)
        fp = 1 if _dtype_code(x) == 0 else 0
        rank = x.ndim
        if axis is None:
            axes = list(range(rank))
        else:
            values = list(axis) if isinstance(axis, (tuple, list)) else [axis]
            axes = [] if (rank == 0 and len(values) == 1 and values[0] in (0, -1)) else values
        out_shape, meta, size = reduction_plan(list(x.shape), axes)
        if not size:
            raise ValueError("min/argmax require a non-empty reduction")
        if code == 4:
            extent = 1
            for a in axes:
                a = a + rank if a < 0 else a
                if x.shape[a] > (2**31 - 1) // extent:
                    raise ValueError("argmax index range exceeds int32")
                extent *= x.shape[a]
        out = np.empty(out_shape, dtype=np.int32 if code == 4 else x.dtype)
        groups = numel(out_shape)
        if groups:
            self.lib.tcxo_min_argmax(code, fp, _ptr(x), _ptr(out), ctypes.c_int64(groups),
                                     ctypes.c_int64(size), _i64(meta), ctypes.c_int64(rank))
        return out

    def min(self, x, axis=None):
        return self._min_argmax(3, x, axis)

    def argmax(self, x, axis=None):
        return self._min_argmax(4, x, axis)

    def philox4x32_10(self, counter, key):
        """The published Philox4x32-10 block function (tcxo_philox4x32_10)."""
        ctr = (ctypes.c_uint32 * 4)(*[int(c) & 0xffffffff for c in counter])
        k = (ctypes.c_uint32 * 2)(*[int(c) & 0xffffffff for c in key])
        out = (ctypes.c_uint32 * 4)()
        self.lib.tcxo_philox4x32_10(ctr, k, out)
        return list(out)

    def random(self, dist, count, seed, offset=0, a=0.0, b=1.0):
        """Checker of tcx_sm100_random: `dist` "normal" (mean a, std b) or "uniform" [a, b)."""
        out = np.empty(count, np.float32)
        self.lib.tcxo_random(ctypes.c_int({"normal": 0, "uniform": 1}[dist]), _ptr(out), ctypes.c_int64(count),
                             ctypes.c_uint64(seed), ctypes.c_uint64(offset), ctypes.c_float(a), ctypes.c_float(b))
        return out

    def sum_f64(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        return float(self.lib.tcxo_sum_f64(_ptr(x), ctypes.c_int64(x.size)))

    # ----------------------------------------------------------------- row ops
    def _rows(self, fn, x, axis, eps=None):
        x = np.ascontiguousarray(x)
        if x.dtype != np.float32:
            raise ValueError("only float32 tensors")
        _, outer, reduce, inner = axis_dims(list(x.shape), axis)
        args = [] if eps is None else [ctypes.c_float(checked_epsilon(eps))]
        out = np.empty_like(x)
        if x.size:
            fn(_ptr(x), _ptr(out), ctypes.c_int64(outer), ctypes.c_int64(reduce),
               ctypes.c_int64(inner), *args)
        return out

    def softmax(self, x, axis=-1):
        return self._rows(self.lib.tcxo_softmax, x, axis)

    def rmsnorm(self, x, axis=-1, eps=1e-5, weight=None):
        out = self._rows(self.lib.tcxo_rmsnorm, x, axis, eps)
        return self._affine(out, axis, weight, None)

    def layernorm(self, x, axis=-1, eps=1e-5, weight=None, bias=None):
        out = self._rows(self.lib.tcxo_layernorm, x, axis, eps)
        return self._affine(out, axis, weight, bias)

    def _affine(self, out, axis, weight, bias):
        """Affine composite of core/inference.cpp:103-122: multiply, then add,
        each a broadcast primitive over the normalized axis."""
        if weight is None and bias is None:
            return out
        shape = [1] * out.ndim
        if out.ndim:
            a = axis + out.ndim if axis < 0 else axis
            shape[a] = out.shape[a]
        if weight is not None:
            out = self.multiply(out, np.asarray(weight, np.float32).reshape(shape))
        if bias is not None:
            out = self.add(out, np.asarray(bias, np.float32).reshape(shape))
        return out

    # -------------------------------------------------------------- elementwise
    def _unary(self, op, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.tcxo_unary(op, _ptr(x), _ptr(out), ctypes.c_int64(x.size))
        return out

    def exp(self, x):
        return self._unary(0, x)

    def gelu(self, x):
        return self._unary(1, x)

    def silu(self, x):
        return self._unary(2, x)

    def _binary(self, op, a, b):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        if a.dtype != b.dtype:
            raise ValueError("dtype mismatch for binary operation")
        dt = _dtype_code(a)
        if op == 3 and dt != 0:
            raise ValueError("division only supports float32 tensors")
        shape, ls, rs = broadcast_plan(list(a.shape), list(b.shape))
        out = np.empty(shape, dtype=a.dtype)
        meta = list(shape) + ls + rs
        if out.size:
            self.lib.tcxo_binary(op, dt, _ptr(a), _ptr(b), _ptr(out), ctypes.c_int64(out.size),
                                 _i64(meta), ctypes.c_int64(len(shape)))
        return out

    def add(self, a, b):
        return self._binary(0, a, b)

    def subtract(self, a, b):
        return self._binary(1, a, b)

    def multiply(self, a, b):
        return self._binary(2, a, b)

    def divide(self, a, b):
        return self._binary(3, a, b)

    def clip(self, x, lower=None, upper=None):
        """python/tensorcx/tensor.py:858-876 then cpu_math.cpp:42-47."""
        x = np.ascontiguousarray(x)
        fp = _dtype_code(x) == 0
        if lower is None and upper is None:
            raise ValueError("clip requires at least one bound")
        lo = np.asarray(lower if lower is not None else (-np.inf if fp else -(2**31)), x.dtype)
        hi = np.asarray(upper if upper is not None else (np.inf if fp else 2**31 - 1), x.dtype)
        shape = list(x.shape)
        for t in (x, lo, hi):
            shape = broadcast_plan(shape, list(t.shape))[0]
        meta = list(shape)
        for t in (x, lo, hi):
            meta += broadcast_plan(list(t.shape), shape)[1]
        out = np.empty(shape, dtype=x.dtype)
        lo, hi = np.ascontiguousarray(lo), np.ascontiguousarray(hi)
        if out.size:
            self.lib.tcxo_clip(int(fp), _ptr(x), _ptr(lo), _ptr(hi), _ptr(out),
                               ctypes.c_int64(out.size), _i64(meta), ctypes.c_int64(len(shape)))
        return out

    def relu(self, x):
        """ReLU as tensor.cx spells it: clip(x, lower=0)."""
        return self.clip(x, 0, None)

    # ------------------------------------------------------------------- matmul
    def matmul(self, a, b, rows=None, batches=None):
        """cpu::matmul over the restated plan. ``rows`` (a slice) and ``batches``
        (an iterable of batch indices) restrict the check to a sample; the
        returned array then holds only those rows of those batches."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        out_shape, bshape, lst, rst, m, k, n = matmul_plan(list(a.shape), list(b.shape))
        nb = numel(bshape) if m and n else 0
        r0, r1 = (0, m) if rows is None else (rows.start, rows.stop)
        sel = list(range(nb)) if batches is None else list(batches)
        out = np.empty((len(sel), r1 - r0, n), dtype=np.float32)
        af, bf = a.reshape(-1), b.reshape(-1)
        for i, bi in enumerate(sel):
            lo = batch_offset(bi, bshape, lst)
            ro = batch_offset(bi, bshape, rst)
            av = np.ascontiguousarray(af[lo:lo + m * k])
            bv = np.ascontiguousarray(bf[ro:ro + k * n])
            ov = out[i]
            if (r1 - r0) and n:
                self.lib.tcxo_matmul_rows(_ptr(av), _ptr(bv), _ptr(ov), ctypes.c_int64(m),
                                          ctypes.c_int64(n), ctypes.c_int64(k),
                                          ctypes.c_int64(r0), ctypes.c_int64(r1))
        if rows is None and batches is None:
            return out.reshape(out_shape)
        return out

    def linear(self, x, w, b=None):
        """core/inference.cpp:89-102: matmul(x, transpose(w)) then add(bias)."""
        y = self.matmul(x, np.ascontiguousarray(np.swapaxes(w, -1, -2)))
        return self.add(y, b) if b is not None else y

    # ---------------------------------------------------------------- attention
    def attention_softmax(self, scores, shape, mask=None, causal=False, scale=1.0):
        """kAttentionSoftmax: cpu_inference.cpp:22-45, with the checks of
        make_attention_softmax_plan (core/inference.cpp:56-83)."""
        scores = np.array(scores, dtype=np.float32, order="C")
        shape = [int(d) for d in shape]
        if scores.ndim < 2 or len(shape) < 2:
            raise ValueError("attention scores must have rank >= 2")
        out_s, sstr, _ = broadcast_plan(list(scores.shape), shape)
        if out_s != shape:
            raise ValueError("attention scores cannot broadcast to target")
        kind, mstr, m = 0, [0] * len(shape), None
        if mask is not None:
            m = np.array(mask, order="C")
            if m.dtype == np.bool_:
                kind, m = 1, m.view(np.uint8)
            elif m.dtype == np.float32:
                kind = 2
            else:
                raise ValueError("attention mask must be bool or float32")
            out_m, mstr, _ = broadcast_plan(list(m.shape), shape)
            if out_m != shape:
                raise ValueError("attention mask cannot broadcast to scores")
        scale = checked_scale(scale)
        out = np.empty(shape, np.float32)
        if out.size:
            self.lib.tcxo_attention_softmax(_ptr(scores), None if m is None else _ptr(m), kind, _ptr(out),
                                            _i64(shape), _i64(sstr), _i64(mstr), len(shape),
                                            ctypes.c_float(scale), int(bool(causal)))
        return out

    def attention(self, q, k, v, mask=None, causal=False, scale=None):
        """kAttention composite (core/inference.cpp:123-160): matmul(q, transpose(k)),
        the attention softmax over the broadcast batch, then matmul with v."""
        q, k, v = (np.array(t, dtype=np.float32, order="C") for t in (q, k, v))
        batch, features = attention_batch(q.shape, k.shape, v.shape)
        scores = list(batch) + [q.shape[-2], k.shape[-2]]
        scale = checked_scale(1.0 / math.sqrt(features) if scale is None else scale)
        product = self.matmul(q, np.ascontiguousarray(np.swapaxes(k, -1, -2)))
        probabilities = self.attention_softmax(product, scores, mask, causal, scale)
        return self.matmul(probabilities, v)


class Reference(_Lib):
    """The reference's own CPU backend (oracle/_ref/libtcx_ref.so)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        self.lib.tcxref_last_error.restype = ctypes.c_char_p

    def _check(self, rc):
        if rc == 1:
            raise ValueError(self.lib.tcxref_last_error().decode())
        if rc != 0:
            raise RuntimeError(self.lib.tcxref_last_error().decode())

    def _unary_op(self, kind, x, axis=0, axes=None, eps=1e-5, out_dtype=None):
        x = np.ascontiguousarray(x)
        dt = _dtype_code(x)
        cap = max(1, x.size)
        out = np.empty(cap, dtype=out_dtype or x.dtype)
        oshape = (ctypes.c_int64 * 64)()
        orank = ctypes.c_int(0)
        naxes = -1 if axes is None else len(axes)
        rc = self.lib.tcxref_unary_op(OPKIND[kind], dt, _ptr(x), _i64(x.shape), x.ndim,
                                      ctypes.c_int64(axis), naxes, _i64(axes or []),
                                      ctypes.c_double(eps), _ptr(out), ctypes.c_int64(cap),
                                      oshape, ctypes.byref(orank))
        self._check(rc)
        shape = [oshape[i] for i in range(orank.value)]
        return out[:numel(shape)].reshape(shape)

    def _reduce(self, name, x, axis):
        mode, sel = axes_for(list(np.shape(x)), axis)
        if mode == "axis":
            return self._unary_op(name, x, axis=sel)
        return self._unary_op(name, x, axes=list(sel))

    def sum(self, x, axis=None):
        return self._reduce("sum", x, axis)

    def max(self, x, axis=None):
        return self._reduce("max", x, axis)

    def mean(self, x, axis=None):
        return self._reduce("mean", x, axis)

    def min(self, x, axis=None):
        rank = np.ndim(x)
        if axis is None:
            axes = list(range(rank))
        else:
            values = list(axis) if isinstance(axis, (tuple, list)) else [axis]
            axes = [] if (rank == 0 and len(values) == 1 and values[0] in (0, -1)) else values
        return self._unary_op("min", x, axes=axes)

    def argmax(self, x, axis=None):
        rank = np.ndim(x)
        if axis is None:
            axes = list(range(rank))
        else:
            axes = [] if (rank == 0 and axis in (0, -1)) else [axis]
        return self._unary_op("argmax", x, axes=axes, out_dtype=np.int32)

    def softmax(self, x, axis=-1):
        return self._unary_op("softmax", x, axis=axis)

    def rmsnorm(self, x, axis=-1, eps=1e-5, weight=None):
        if weight is None:
            return self._unary_op("rmsnorm", x, axis=axis, eps=eps)
        return self._affine(1, x, axis, eps, weight, None)

    def layernorm(self, x, axis=-1, eps=1e-5, weight=None, bias=None):
        if weight is None and bias is None:
            return self._unary_op("layernorm", x, axis=axis, eps=eps)
        return self._affine(0, x, axis, eps, weight, bias)

    def _affine(self, rms, x, axis, eps, weight, bias):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        w = None if weight is None else np.ascontiguousarray(weight, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        rc = self.lib.tcxref_affine_norm(rms, _ptr(x), _i64(x.shape), x.ndim,
                                         ctypes.c_int64(axis), ctypes.c_double(eps),
                                         None if w is None else _ptr(w),
                                         None if b is None else _ptr(b), _ptr(out),
                                         ctypes.c_int64(max(1, x.size)))
        self._check(rc)
        return out

    def exp(self, x):
        return self._unary_op("exp", x)

    def gelu(self, x):
        return self._unary_op("gelu", x)

    def silu(self, x):
        return self._unary_op("silu", x)

    def _binary(self, kind, a, b, cap=None):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        dt = _dtype_code(a) if a.dtype == b.dtype else -1
        if dt < 0:
            raise ValueError("dtype mismatch for binary operation")
        cap = cap or max(1, a.size * max(1, b.size))
        out = np.empty(cap, dtype=a.dtype)
        oshape = (ctypes.c_int64 * 64)()
        orank = ctypes.c_int(0)
        rc = self.lib.tcxref_binary_op(OPKIND[kind], dt, _ptr(a), _i64(a.shape), a.ndim,
                                       _ptr(b), _i64(b.shape), b.ndim, _ptr(out),
                                       ctypes.c_int64(cap), oshape, ctypes.byref(orank))
        self._check(rc)
        shape = [oshape[i] for i in range(orank.value)]
        return out[:numel(shape)].reshape(shape)

    def add(self, a, b):
        return self._binary("add", a, b)

    def subtract(self, a, b):
        return self._binary("subtract", a, b)

    def multiply(self, a, b):
        return self._binary("multiply", a, b)

    def divide(self, a, b):
        return self._binary("divide", a, b)

    def matmul(self, a, b):
        a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
        out_shape = matmul_plan(list(a.shape), list(b.shape))[0]
        return self._binary("matmul", a, b, cap=max(1, numel(out_shape)))

    def matmul_bind_rhs(self, b):
        """Copy B into the reference's CpuTensor once; later matmul_rows calls on the
        same (contiguous float32) B use that copy instead of copying B per call."""
        assert b.dtype == np.float32 and b.flags.c_contiguous
        self._check(self.lib.tcxref_matmul_bind_rhs(_ptr(b), ctypes.c_int64(b.shape[0]),
                                                    ctypes.c_int64(b.shape[1])))

    def matmul_rows(self, a, b, row_begin, row_end):
        """cpu::matmul on a row slice of a 2-D lhs (same per-element arithmetic)."""
        m, k = a.shape
        n = b.shape[1]
        out = np.empty((row_end - row_begin, n), np.float32)
        rc = self.lib.tcxref_matmul_rows(_ptr(a), _ptr(b), _ptr(out), ctypes.c_int64(m),
                                         ctypes.c_int64(k), ctypes.c_int64(n),
                                         ctypes.c_int64(row_begin), ctypes.c_int64(row_end))
        self._check(rc)
        return out

    def clip(self, x, lower=None, upper=None):
        x = np.ascontiguousarray(x)
        fp = x.dtype == np.float32
        lo = np.ascontiguousarray(np.asarray(lower if lower is not None else (-np.inf if fp else -(2**31)), x.dtype))
        hi = np.ascontiguousarray(np.asarray(upper if upper is not None else (np.inf if fp else 2**31 - 1), x.dtype))
        cap = max(1, x.size, lo.size, hi.size) * 4
        out = np.empty(cap, dtype=x.dtype)
        oshape = (ctypes.c_int64 * 64)()
        orank = ctypes.c_int(0)
        rc = self.lib.tcxref_clip(_dtype_code(x), _ptr(x), _i64(x.shape), x.ndim, _ptr(lo),
                                  _i64(lo.shape), lo.ndim, _ptr(hi), _i64(hi.shape), hi.ndim,
                                  _ptr(out), ctypes.c_int64(cap), oshape, ctypes.byref(orank))
        self._check(rc)
        shape = [oshape[i] for i in range(orank.value)]
        return out[:numel(shape)].reshape(shape)

    def relu(self, x):
        return self.clip(x, 0, None)

    def linear(self, x, w, b=None):
        x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
        shape = list(x.shape[:-1]) + [w.shape[0]]
        out = np.empty(max(1, numel(shape)), np.float32)
        bb = None if b is None else np.ascontiguousarray(b, np.float32)
        rc = self.lib.tcxref_linear(_ptr(x), _i64(x.shape), x.ndim, _ptr(w), _i64(w.shape),
                                    None if bb is None else _ptr(bb), _ptr(out),
                                    ctypes.c_int64(out.size))
        self._check(rc)
        return out[:numel(shape)].reshape(shape)

    def attention(self, q, k, v, mask=None, causal=False, scale=None):
        q, k, v = (np.array(t, dtype=np.float32, order="C") for t in (q, k, v))
        kind, m = 0, None
        if mask is not None:
            m = np.array(mask, order="C")
            kind = 1 if m.dtype == np.bool_ else 2
            if kind == 1:
                m = m.view(np.uint8)
        try:
            batch = np.broadcast_shapes(q.shape[:-2], k.shape[:-2], v.shape[:-2])
            cap = max(1, int(np.prod(batch, dtype=np.int64)) * q.shape[-2] * v.shape[-1])
        except ValueError:
            cap = 1
        out = np.empty(cap, np.float32)
        oshape = (ctypes.c_int64 * 64)()
        orank = ctypes.c_int(0)
        rc = self.lib.tcxref_attention(_ptr(q), _i64(q.shape), q.ndim, _ptr(k), _i64(k.shape), k.ndim,
                                       _ptr(v), _i64(v.shape), v.ndim, None if m is None else _ptr(m), kind,
                                       _i64([] if m is None else m.shape), 0 if m is None else m.ndim,
                                       int(bool(causal)), int(scale is not None),
                                       ctypes.c_double(0.0 if scale is None else scale), _ptr(out),
                                       ctypes.c_int64(cap), oshape, ctypes.byref(orank))
        self._check(rc)
        shape = [oshape[i] for i in range(orank.value)]
        return out[:numel(shape)].reshape(shape)

    def attention_softmax(self, scores, shape, mask=None, causal=False, scale=1.0):
        scores = np.array(scores, dtype=np.float32, order="C")
        kind, m = 0, None
        if mask is not None:
            m = np.array(mask, order="C")
            kind = 1 if m.dtype == np.bool_ else 2
            if kind == 1:
                m = m.view(np.uint8)
        cap = max(1, numel(list(shape)))
        out = np.empty(cap, np.float32)
        rc = self.lib.tcxref_attention_softmax(_ptr(scores), _i64(scores.shape), scores.ndim,
                                               None if m is None else _ptr(m), kind,
                                               _i64([] if m is None else m.shape), 0 if m is None else m.ndim,
                                               _i64(list(shape)), len(shape), int(bool(causal)),
                                               ctypes.c_double(scale), _ptr(out), ctypes.c_int64(cap))
        self._check(rc)
        return out[:numel(list(shape))].reshape(list(shape))
