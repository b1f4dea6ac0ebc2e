"""Python host mirror of the tensor.cx op API for device='cuda' on B200.

Names, argument meaning and errors follow python/tensorcx/tensor.py (matmul 500-505,
sum/max/mean 508-545, softmax/rmsnorm/layernorm 565-584, min/argmax 834-855,
clip 858-876) and the primitive dispatch of CudaBackend::execute
(cpp/tensorcx/backends/cuda/cuda_backend.cpp:290-627). Tensors are torch CUDA tensors
(float32 or int32, contiguous): torch supplies device memory and streams, nothing else.
Every op calls the C ABI (tensorcx_b200._abi) on torch's current stream; outputs are
fresh contiguous tensors, and workspace comes from torch's stream-ordered caching
allocator. Ops are asynchronous like torch ops; call torch.cuda.synchronize() (or
.cpu()) to observe results.
"""
from __future__ import annotations

import builtins
import ctypes
import math
import operator

import numpy as np
import torch

from . import plan
from ._abi import ACT, FLOAT32, INT32, MATMUL_PATH, OP, Partial, check, i64_array, lib

__all__ = ["matmul", "sum", "max", "mean", "min", "argmax", "softmax", "rmsnorm", "layernorm",
           "exp", "gelu", "silu", "add", "subtract", "multiply", "divide", "clip", "relu",
           "bias_act", "linear", "attention", "scaled_dot_product_attention", "attention_softmax",
           "reduce_partial", "reduce_combine", "Partial", "randn", "rand_uniform"]


def _dtype(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return FLOAT32
    if t.dtype == torch.int32:
        return INT32
    raise ValueError("CUDA operations only support float32 and int32 on this path")


def _check_tensor(t: torch.Tensor, name: str = "input") -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise ValueError("device mismatch: tensors must be on the CUDA device")
    # the kernels launch on the current device's stream: a tensor of another GPU would be
    # read there through its device address
    if t.device.index is not None and t.device.index != torch.cuda.current_device():
        raise ValueError(f"device mismatch: {name} is on {t.device} but the current device is "
                         f"cuda:{torch.cuda.current_device()} (use torch.cuda.device)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream() -> ctypes.c_void_p:
    """torch's current stream on the current device (the raw handle, without building a
    torch.cuda.Stream object: ~0.2 us instead of ~3 us per op)."""
    if _raw_stream is not None:
        return ctypes.c_void_p(_raw_stream(torch.cuda.current_device()))
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _workspace(nbytes: int, device, align: int = 1024):
    """(keep-alive tensor, aligned pointer) for `nbytes` of scratch, or (None, None)."""
    if nbytes == 0:
        return None, None
    buf = torch.empty(nbytes + align, dtype=torch.uint8, device=device)
    addr = (buf.data_ptr() + align - 1) // align * align
    return buf, ctypes.c_void_p(addr)


# -------------------------------------------------------------------- matmul
_matmul_plans: dict = {}


def _matmul_plan(lhs_shape, rhs_shape):
    """make_matmul_plan for a shape pair with its ctypes metadata arrays, cached (a
    failing plan raises each time and is not cached)."""
    key = (tuple(lhs_shape), tuple(rhs_shape))
    hit = _matmul_plans.get(key)
    if hit is None:
        p = plan.matmul(lhs_shape, rhs_shape)
        hit = (p, i64_array(p.batch_shape), i64_array(p.lhs_batch_strides), i64_array(p.rhs_batch_strides))
        if len(_matmul_plans) > 4096:
            _matmul_plans.clear()
        _matmul_plans[key] = hit
    return hit


def matmul(lhs: torch.Tensor, rhs: torch.Tensor, *, bias: torch.Tensor | None = None,
           act: str = "none", path: str = "auto", out: torch.Tensor | None = None) -> torch.Tensor:
    """NumPy-semantics float32 matmul; optional fused epilogue act(C + bias[n])."""
    _check_tensor(lhs, "lhs"), _check_tensor(rhs, "rhs")
    if lhs.device != rhs.device:
        raise ValueError("device mismatch for matmul")
    if lhs.dtype != torch.float32 or rhs.dtype != torch.float32:
        raise ValueError("matmul only supports float32 tensors")
    p, shape_a, lstr_a, rstr_a = _matmul_plan(lhs.shape, rhs.shape)
    if out is None:
        out = torch.empty(p.output_shape, dtype=torch.float32, device=lhs.device)
    else:
        # the kernels write every element of out and read the operands while doing so
        _check_tensor(out, "out")
        if out.device != lhs.device or out.dtype != torch.float32 or tuple(out.shape) != tuple(p.output_shape):
            raise ValueError(f"out must be a float32 tensor of shape {tuple(p.output_shape)} on {lhs.device}")
        for t in (lhs, rhs):
            if t.numel() and out.numel() and out.data_ptr() < t.data_ptr() + t.numel() * 4 and \
                    t.data_ptr() < out.data_ptr() + out.numel() * 4:
                raise ValueError("out must not overlap the operands")
    if bias is not None:
        _check_tensor(bias, "bias")
        if bias.shape != (p.n,) or bias.dtype != torch.float32:
            raise ValueError("bias must be float32 with shape (n,)")
    nba = lhs.numel() // builtins.max(1, p.m * p.k) if p.m * p.k else 1
    nbb = rhs.numel() // builtins.max(1, p.k * p.n) if p.k * p.n else 1
    ws_bytes = lib().tcx_sm100_matmul_workspace_bytes(p.m, p.n, p.k, nba, nbb, MATMUL_PATH[path])
    keep, ws = _workspace(ws_bytes, lhs.device)
    batches = plan.numel(p.batch_shape) if out.numel() else 0
    check(lib().tcx_sm100_matmul(
        _stream(), _ptr(lhs), _ptr(rhs), _ptr(out), p.m, p.n, p.k, batches,
        shape_a, lstr_a, rstr_a, len(p.batch_shape), _ptr(bias), ACT[act], MATMUL_PATH[path], ws, ws_bytes))
    del keep
    return out


def matmul_host(a_host: torch.Tensor, b_host: torch.Tensor, c_host: torch.Tensor | None = None,
                device: int | None = None) -> torch.Tensor:
    """C = A @ B for 2-D float32 HOST tensors (pinned for copy/compute overlap):
    tcx_sm100_matmul_host pipelines the uploads, GEMMs and downloads in row chunks.
    Returns the host tensor C (synchronous)."""
    for t, name in ((a_host, "lhs"), (b_host, "rhs")):
        if not isinstance(t, torch.Tensor) or t.is_cuda or t.dtype != torch.float32 or t.dim() != 2:
            raise ValueError(f"{name} must be a 2-D float32 host tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    m, k = a_host.shape
    if b_host.shape[0] != k:
        raise ValueError("matmul shape mismatch: contracting dimensions differ")
    n = b_host.shape[1]
    if c_host is None:
        c_host = torch.empty((m, n), dtype=torch.float32, pin_memory=a_host.is_pinned())
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        ws_bytes = lib().tcx_sm100_matmul_host_workspace_bytes(m, n, k)
        keep, ws = _workspace(ws_bytes, dev)
        torch.cuda.current_stream().synchronize()  # workspace allocation is stream-ordered
        check(lib().tcx_sm100_matmul_host(_ptr(a_host), _ptr(b_host), _ptr(c_host), m, n, k, ws, ws_bytes))
    del keep
    return c_host


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           act: str = "none", path: str = "auto") -> torch.Tensor:
    """linear(x[..., in], w[out, in], b[out]) (core/inference.cpp:89-102) as one GEMM:
    the weight is read in place (K-major), the bias and optional activation run in the
    epilogue; no transpose copy, no separate add."""
    _check_tensor(x, "x"), _check_tensor(weight, "weight")
    if x.dtype != torch.float32 or weight.dtype != torch.float32:
        raise ValueError("inference values require float32 tensors")
    if x.dim() == 0 or weight.dim() != 2 or x.shape[-1] != weight.shape[1]:
        raise ValueError("linear requires (..., in_features) and (out_features, in_features)")
    if bias is not None:
        _check_tensor(bias, "bias")
        if tuple(bias.shape) != (weight.shape[0],):
            raise ValueError("linear bias must have shape (out_features,)")
    rows = x.numel() // x.shape[-1] if x.shape[-1] else plan.numel(x.shape[:-1])
    out = torch.empty(tuple(x.shape[:-1]) + (weight.shape[0],), dtype=torch.float32, device=x.device)
    ws_bytes = lib().tcx_sm100_linear_workspace_bytes(rows, weight.shape[1], weight.shape[0], MATMUL_PATH[path])
    keep, ws = _workspace(ws_bytes, x.device)
    check(lib().tcx_sm100_linear(_stream(), _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), rows, weight.shape[1],
                                 weight.shape[0], ACT[act], MATMUL_PATH[path], ws, ws_bytes))
    del keep
    return out


# ---------------------------------------------------------------- reductions
def _normalize_axis(axis) -> int:
    """tensor.py:422-431: an operator.index integer, never a bool."""
    if isinstance(axis, (bool, np.bool_)):
        raise ValueError("axis must be an integer")
    try:
        value = operator.index(axis)
    except TypeError:
        raise ValueError("axis must be an integer") from None
    if value < -(2**63) or value > 2**63 - 1:
        raise ValueError("axis is out of range")
    return int(value)


def _axis_sequence(axes) -> tuple[tuple[int, ...], bool]:
    """tensor.py:279-292: integer axes and whether the argument was one integer."""
    if isinstance(axes, (bool, np.bool_, str, bytes)):
        raise ValueError("axis must be an integer or iterable of integers")
    try:
        value = operator.index(axes)
    except TypeError:
        try:
            values = tuple(axes)
        except TypeError:
            raise ValueError("axis must be an integer or iterable of integers") from None
        return tuple(_normalize_axis(v) for v in values), False
    return (_normalize_axis(value),), True


def _axes_in_rank(axes, rank: int, label: str = "reduction axis") -> tuple[int, ...]:
    """tensor.py:295-301: in range after wrapping negatives, no repeats."""
    normalized = tuple(a + rank if a < 0 else a for a in axes)
    if builtins.any(a < 0 or a >= rank for a in normalized):
        raise ValueError(f"{label} is out of range")
    if len(set(normalized)) != len(normalized):
        raise ValueError("axes must not repeat")
    return normalized


def _check_keepdims(keepdims) -> None:
    if not isinstance(keepdims, (bool, np.bool_)):
        raise TypeError("keepdims must be a boolean")


def _keep(result: torch.Tensor, x: torch.Tensor, axes, keepdims) -> torch.Tensor:
    """tensor.py:526-529: reduced axes come back as extent 1 (a view, no copy)."""
    if keepdims and x.dim():
        selected = set(axes)
        return result.reshape(tuple(1 if i in selected else n for i, n in enumerate(x.shape)))
    return result


def _reduce(name: str, x: torch.Tensor, axis, keepdims=False) -> torch.Tensor:
    """tensor.py:508-529: a single axis (or a scalar's 0/-1) uses the one-axis
    primitive, every other selection (None = all axes) the multi-axis plan."""
    _check_tensor(x)
    _check_keepdims(keepdims)
    dt = _dtype(x)
    if name == "mean" and dt != FLOAT32:
        raise ValueError("mean only supports float32 tensors")
    rank = x.dim()
    if axis is None:
        axes, scalar = tuple(range(rank)), rank == 0
    else:
        values, single = _axis_sequence(axis)
        scalar = rank == 0 and single and values[0] in (0, -1)
        axes = () if scalar else _axes_in_rank(values, rank)
    if scalar or len(axes) == 1:
        shape, outer, reduce, inner = plan.axis(list(x.shape), axes[0] if axes else 0)
        if name == "max" and reduce == 0:
            raise ValueError("max reduction requires a non-empty axis")
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
        ws_bytes = lib().tcx_sm100_axis_workspace_bytes(OP[name], outer, reduce, inner)
        keep, ws = _workspace(ws_bytes, x.device)
        check(lib().tcx_sm100_axis(_stream(), OP[name], dt, _ptr(x), _ptr(out), outer, reduce, inner,
                                   0.0, ws, ws_bytes))
        return _keep(out, x, axes, keepdims)
    p = plan.reduction(list(x.shape), axes)
    if name == "max" and p.reduction_size == 0:
        raise ValueError("max reduction requires non-empty axes")
    if not axes:
        return x.clone()
    out = torch.empty(p.output_shape, dtype=x.dtype, device=x.device)
    groups = plan.numel(p.output_shape)
    ws_bytes = lib().tcx_sm100_reduce_workspace_bytes(groups * p.reduction_size)
    keep, ws = _workspace(ws_bytes, x.device)
    check(lib().tcx_sm100_reduce_axes(_stream(), OP[name], dt, _ptr(x), _ptr(out), groups,
                                      p.reduction_size, i64_array(p.index_metadata),
                                      len(p.output_shape), x.dim(), ws, ws_bytes))
    return _keep(out, x, axes, keepdims)


def sum(x: torch.Tensor, axis=None, keepdims=False) -> torch.Tensor:  # noqa: A001 - tensor.cx name
    return _reduce("sum", x, axis, keepdims)


def max(x: torch.Tensor, axis=None, keepdims=False) -> torch.Tensor:  # noqa: A001
    return _reduce("max", x, axis, keepdims)


def mean(x: torch.Tensor, axis=None, keepdims=False) -> torch.Tensor:
    return _reduce("mean", x, axis, keepdims)


def _min_argmax(name: str, x: torch.Tensor, axis, keepdims=False) -> torch.Tensor:
    """tensor.py:834-855 (min takes any axis selection, argmax one axis or None),
    make_math_plan (core/math.cpp:39-56), then the C ABI."""
    _check_tensor(x)
    _check_keepdims(keepdims)
    dt = _dtype(x)
    rank = x.dim()
    if axis is None:
        axes = tuple(range(rank))
    elif name == "argmax":
        value = _normalize_axis(axis)
        axes = () if rank == 0 and value in (0, -1) else _axes_in_rank((value,), rank, "axis")
    else:
        values, single = _axis_sequence(axis)
        scalar = rank == 0 and single and values[0] in (0, -1)
        axes = () if scalar else _axes_in_rank(values, rank)
    p = plan.reduction(list(x.shape), axes)
    if not p.reduction_size:
        raise ValueError("min/argmax require a non-empty reduction")
    if name == "argmax":
        extent = 1
        for a in axes:
            if x.shape[a] > (2**31 - 1) // extent:
                raise ValueError("argmax index range exceeds int32")
            extent *= x.shape[a]
    out = torch.empty(p.output_shape, dtype=torch.int32 if name == "argmax" else x.dtype, device=x.device)
    groups = plan.numel(p.output_shape)
    ws_bytes = lib().tcx_sm100_reduce_workspace_bytes(groups * p.reduction_size)
    keep, ws = _workspace(ws_bytes, x.device)
    check(lib().tcx_sm100_min_argmax(_stream(), OP[name], dt, _ptr(x), _ptr(out), groups,
                                     p.reduction_size, i64_array(p.index_metadata), x.dim(), ws,
                                     ws_bytes))
    return _keep(out, x, axes, keepdims)


def min(x: torch.Tensor, axis=None, keepdims=False) -> torch.Tensor:  # noqa: A001
    return _min_argmax("min", x, axis, keepdims)


def argmax(x: torch.Tensor, axis=None, keepdims=False) -> torch.Tensor:
    return _min_argmax("argmax", x, axis, keepdims)


def reduce_partial(x: torch.Tensor, op: str, index_base: int = 0) -> torch.Tensor:
    """This shard's 16-byte tcx_partial record (as a uint8[16] device tensor) for a
    full-tensor reduction combined across GPUs with reduce_combine."""
    _check_tensor(x)
    rec = torch.empty(16, dtype=torch.uint8, device=x.device)
    ws_bytes = lib().tcx_sm100_reduce_workspace_bytes(x.numel())
    keep, ws = _workspace(ws_bytes, x.device)
    check(lib().tcx_sm100_reduce_partial(_stream(), OP[op], _dtype(x), _ptr(x), x.numel(), index_base,
                                         _ptr(rec), ws, ws_bytes))
    return rec


def reduce_combine(records: torch.Tensor, op: str, dtype: torch.dtype, total_count: int) -> torch.Tensor:
    """Folds gathered records ([nparts, 16] uint8, rank order) into the final value."""
    out = torch.empty((), dtype=torch.int32 if op == "argmax" else dtype, device=records.device)
    dt = FLOAT32 if dtype == torch.float32 else INT32
    check(lib().tcx_sm100_reduce_combine(_stream(), OP[op], dt, _ptr(records.contiguous()),
                                         records.numel() // 16, total_count, _ptr(out)))
    return out


# ------------------------------------------------------------------ row ops
def _row_op(name: str, x: torch.Tensor, axis: int, eps: float | None, weight=None, bias=None):
    _check_tensor(x)
    if x.dtype != torch.float32:
        raise ValueError(f"{name} only supports float32 tensors")
    _, outer, reduce, inner = plan.axis(list(x.shape), axis)
    e = plan.epsilon(eps) if eps is not None else 0.0
    out = torch.empty_like(x)
    if weight is None and bias is None:
        check(lib().tcx_sm100_axis(_stream(), OP[name], FLOAT32, _ptr(x), _ptr(out), outer, reduce, inner,
                                   e, None, 0))
        return out
    expected = () if x.dim() == 0 else (reduce,)
    for t in (weight, bias):
        if t is not None:
            _check_tensor(t)
            if tuple(t.shape) != expected or t.dtype != torch.float32:
                raise ValueError("affine parameters must match the normalized axis")
    check(lib().tcx_sm100_affine_norm(_stream(), OP[name], _ptr(x), _ptr(out), outer, reduce, inner, e,
                                      _ptr(weight), _ptr(bias)))
    return out


def softmax(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    return _row_op("softmax", x, axis, None)


def rmsnorm(x: torch.Tensor, axis: int = -1, eps: float = 1.0e-5, *, weight=None) -> torch.Tensor:
    return _row_op("rmsnorm", x, axis, eps, weight, None)


def layernorm(x: torch.Tensor, axis: int = -1, eps: float = 1.0e-5, *, weight=None, bias=None) -> torch.Tensor:
    return _row_op("layernorm", x, axis, eps, weight, bias)


# -------------------------------------------------------------- elementwise
def _unary(name: str, x: torch.Tensor) -> torch.Tensor:
    _check_tensor(x)
    if x.dtype != torch.float32:
        raise ValueError(f"{name} only supports float32 tensors")
    out = torch.empty_like(x)
    check(lib().tcx_sm100_unary(_stream(), OP[name], _ptr(x), _ptr(out), x.numel()))
    return out


def exp(x):
    return _unary("exp", x)


def gelu(x):
    return _unary("gelu", x)


def silu(x):
    return _unary("silu", x)


def _binary(name: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    _check_tensor(a), _check_tensor(b)
    if a.dtype != b.dtype:
        raise ValueError("dtype mismatch for binary operation")
    dt = _dtype(a)
    if name == "divide" and dt != FLOAT32:
        raise ValueError("division only supports float32 tensors")
    shape, ls, rs = plan.broadcast(list(a.shape), list(b.shape))
    out = torch.empty(shape, dtype=a.dtype, device=a.device)
    same = list(a.shape) == list(b.shape)
    meta = [] if same else list(shape) + ls + rs
    check(lib().tcx_sm100_binary(_stream(), OP[name], dt, _ptr(a), _ptr(b), _ptr(out), out.numel(),
                                 i64_array(meta) if meta else None, 0 if same else len(shape)))
    return out


def add(a, b):
    return _binary("add", a, b)


def subtract(a, b):
    return _binary("subtract", a, b)


def multiply(a, b):
    return _binary("multiply", a, b)


def divide(a, b):
    return _binary("divide", a, b)


def clip(x: torch.Tensor, lower=None, upper=None) -> torch.Tensor:
    """tensor.py:858-876: scalar or tensor bounds, None leaves that side open."""
    _check_tensor(x)
    dt = _dtype(x)
    if lower is None and upper is None:
        raise ValueError("clip requires at least one bound")
    bounds = []
    for i, v in enumerate((lower, upper)):
        if v is None:
            v = (-math.inf if i == 0 else math.inf) if dt == FLOAT32 else (-(2**31) if i == 0 else 2**31 - 1)
        if not isinstance(v, torch.Tensor):
            v = torch.tensor(v, dtype=x.dtype, device=x.device)
        if v.dtype != x.dtype:
            raise ValueError("clip input dtypes must match")
        bounds.append(v.contiguous())
    shape = list(x.shape)
    for t in (x, *bounds):
        shape = plan.broadcast(shape, list(t.shape))[0]
    meta = list(shape)
    for t in (x, *bounds):
        meta += plan.broadcast(list(t.shape), shape)[1]
    out = torch.empty(shape, dtype=x.dtype, device=x.device)
    check(lib().tcx_sm100_clip(_stream(), dt, _ptr(x), _ptr(bounds[0]), _ptr(bounds[1]), _ptr(out),
                               out.numel(), i64_array(meta), len(shape)))
    return out


def relu(x: torch.Tensor) -> torch.Tensor:
    """ReLU as tensor.cx spells it: clip(x, lower=0)."""
    return clip(x, 0, None)


def bias_act(x: torch.Tensor, bias: torch.Tensor | None, act: str = "silu") -> torch.Tensor:
    """Fused chain act(x + bias[-1 axis]) in one pass (the add + activation pair)."""
    _check_tensor(x)
    cols = x.shape[-1] if x.dim() else 1
    if bias is not None:
        _check_tensor(bias, "bias")
        if tuple(bias.shape) != (cols,):
            raise ValueError("bias must match the last axis")
    out = torch.empty_like(x)
    rows = x.numel() // cols if cols else 0
    check(lib().tcx_sm100_bias_act(_stream(), _ptr(x), _ptr(bias), _ptr(out), rows, cols, ACT[act]))
    return out


# ---------------------------------------------------------------- attention
def _checked_scale(scale: float) -> float:
    """checked_scale (core/inference.cpp:15-20): finite, representable as float32 and
    not flushed to zero."""
    finite = math.isfinite(scale)
    narrowed = float(np.float32(scale)) if finite and abs(scale) <= 3.4028234663852886e38 else math.inf
    if not finite or not math.isfinite(narrowed) or (scale != 0 and narrowed == 0):
        raise ValueError("attention scale must be finite and representable as float32")
    return narrowed


def _broadcast_strides(shape, target):
    """Element strides of a contiguous `shape` read as broadcast to `target` (0 on
    broadcast axes), or None when it does not broadcast (shape.cpp:78-104)."""
    rank, own = len(target), len(shape)
    if own > rank:
        return None
    contiguous = plan.strides(list(shape))
    out = [0] * rank
    for a in range(rank):
        if a < rank - own:
            continue
        d = shape[a - (rank - own)]
        if d != target[a] and d != 1:
            return None
        if d != 1:
            out[a] = contiguous[a - (rank - own)]
    return out


def _mask_kind(mask: torch.Tensor) -> int:
    if mask.dtype == torch.bool:
        return 1
    if mask.dtype == torch.float32:
        return 2
    raise ValueError("attention mask must be bool or float32")


def attention_softmax(scores: torch.Tensor, shape=None, mask: torch.Tensor | None = None, *, scale: float = 1.0,
                      is_causal: bool = False) -> torch.Tensor:
    """The kAttentionSoftmax primitive (core/inference.cpp:56-83): softmax over the
    last axis of scale * scores + mask, scores and mask broadcast to `shape`
    (default: the scores' shape), masked entries -inf, fully masked rows zero."""
    _check_tensor(scores, "scores")
    if scores.dtype != torch.float32:
        raise ValueError("inference values require float32 tensors")
    target = list(scores.shape) if shape is None else [int(d) for d in shape]
    if scores.dim() < 2 or len(target) < 2:
        raise ValueError("attention scores must have rank >= 2")
    sstr = _broadcast_strides(list(scores.shape), target)
    if sstr is None:
        raise ValueError("attention scores cannot broadcast to target")
    kind, mstr = 0, None
    if mask is not None:
        _check_tensor(mask, "mask")
        kind = _mask_kind(mask)
        mstr = _broadcast_strides(list(mask.shape), target)
        if mstr is None:
            raise ValueError("attention mask cannot broadcast to scores")
    s = _checked_scale(float(scale))
    plan.numel(target)
    out = torch.empty(target, dtype=torch.float32, device=scores.device)
    check(lib().tcx_sm100_attention_softmax(_stream(), _ptr(scores), _ptr(mask), kind, _ptr(out),
                                            i64_array(target), i64_array(sstr),
                                            i64_array(mstr) if mstr is not None else None, len(target), s,
                                            int(bool(is_causal))))
    return out


def scaled_dot_product_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                 attn_mask: torch.Tensor | None = None, *, is_causal=False,
                                 scale=None) -> torch.Tensor:
    """tensor.py:924-946 and the kAttention composite (core/inference.cpp:123-160):
    softmax(scale * query·keyᵀ + mask) · value over broadcast batch dimensions; True
    mask entries are allowed, causal is upper-left, the default scale 1/sqrt(features).
    Runs as one C-ABI call: without a mask (and with feature sizes that are multiples of
    32 up to 128) one fused tcgen05 kernel, otherwise two tcgen05 GEMMs (keys read
    K-major, no transpose copy) around the masked softmax."""
    tensors = (query, key, value) + (() if attn_mask is None else (attn_mask,))
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError("attention expects Tensor arguments")
    if builtins.any(t.device != query.device for t in tensors):
        raise ValueError("device mismatch: attention tensors must share one device")
    if not isinstance(is_causal, (bool, np.bool_)):
        raise TypeError("is_causal must be a boolean")
    if scale is not None:
        if isinstance(scale, (bool, np.bool_)) or not isinstance(scale, (int, float, np.integer, np.floating)):
            raise TypeError("attention scale must be a real scalar")
        try:
            scale = float(scale)
        except OverflowError:
            raise ValueError("attention scale is out of range") from None
    for t in (query, key, value):
        _check_tensor(t)
        if t.dtype != torch.float32:
            raise ValueError("inference values require float32 tensors")
        if t.dim() < 2:
            raise ValueError("attention tensors require rank >= 2")
    features, queries, keys = query.shape[-1], query.shape[-2], key.shape[-2]
    if features <= 0 or features != key.shape[-1] or keys != value.shape[-2]:
        raise ValueError("attention query/key features and key/value sequence sizes must match; "
                         "features must be positive")
    batch = []
    for t in (query, key, value):
        own = list(t.shape[:-2])
        rank = builtins.max(len(batch), len(own))
        merged = []
        for a in range(rank):
            left = 1 if a < rank - len(batch) else batch[a - (rank - len(batch))]
            right = 1 if a < rank - len(own) else own[a - (rank - len(own))]
            if left != right and left != 1 and right != 1:
                raise ValueError("attention batch dimensions cannot broadcast")
            merged.append(right if left == 1 else left)
        batch = merged
    scores_shape = batch + [queries, keys]
    out_shape = batch + [queries, value.shape[-1]]
    plan.numel(scores_shape), plan.numel(out_shape)
    s = _checked_scale(1.0 / math.sqrt(features) if scale is None else scale)
    kind, mstr = 0, None
    if attn_mask is not None:
        _check_tensor(attn_mask, "mask")
        kind = _mask_kind(attn_mask)
        mstr = _broadcast_strides(list(attn_mask.shape), scores_shape)
        if mstr is None:
            raise ValueError("attention mask cannot broadcast to scores")
    out = torch.empty(out_shape, dtype=torch.float32, device=query.device)
    if out.numel() == 0:
        return out
    rank = len(batch)

    def batch_strides(t):
        st = _broadcast_strides(list(t.shape), batch + list(t.shape[-2:]))
        return st[:rank]
    qs, ks, vs = batch_strides(query), batch_strides(key), batch_strides(value)
    nb = plan.numel(batch)
    ws_bytes = lib().tcx_sm100_attention_workspace_bytes(
        nb, queries, keys, features, value.shape[-1], plan.numel(list(query.shape[:-2])),
        plan.numel(list(key.shape[:-2])), plan.numel(list(value.shape[:-2])), kind)
    keep, ws = _workspace(ws_bytes, query.device)
    check(lib().tcx_sm100_attention(_stream(), _ptr(query), _ptr(key), _ptr(value), _ptr(attn_mask), kind,
                                    _ptr(out), queries, keys, features, value.shape[-1], i64_array(batch),
                                    i64_array(qs), i64_array(ks), i64_array(vs), rank,
                                    i64_array(mstr) if mstr is not None else None, s, int(bool(is_causal)),
                                    ws, ws_bytes))
    del keep
    return out


attention = scaled_dot_product_attention


# -------------------------------------------------------------------- generation
def _shape_of(shape) -> tuple[int, ...]:
    dims = (shape,) if isinstance(shape, (int, np.integer)) else tuple(shape)
    out = []
    for d in dims:
        if isinstance(d, (bool, np.bool_)) or not isinstance(d, (int, np.integer)):
            raise TypeError("shape dimensions must be integers")
        if d < 0:
            raise ValueError("shape dimensions must be non-negative")
        out.append(int(d))
    return tuple(out)


def _seed_of(seed) -> int:
    if seed is None:
        import secrets
        return secrets.randbits(64)
    if isinstance(seed, (bool, np.bool_)) or not isinstance(seed, (int, np.integer)) or not 0 <= seed < 2**64:
        raise ValueError("seed must be an integer in [0, 2**64)")
    return int(seed)


def _generate(kind: int, shape, seed, offset: int, a: float, b: float, device) -> torch.Tensor:
    dims = _shape_of(shape)
    if isinstance(offset, (bool, np.bool_)) or not isinstance(offset, (int, np.integer)) or offset < 0:
        raise ValueError("offset must be a non-negative integer")
    s = _seed_of(seed)
    out = torch.empty(dims, dtype=torch.float32, device=device)
    if not out.is_cuda:
        raise ValueError("generation targets a CUDA device")
    check(lib().tcx_sm100_random(_stream(), kind, _ptr(out), out.numel(), s, int(offset), a, b))
    return out


def randn(shape, dtype: str = "float32", device="cuda", seed: int | None = None, *, offset: int = 0) -> torch.Tensor:
    """tensor.cx's randn (python/tensorcx/tensor.py:485-497) made on the device:
    standard normal float32 from the counter-based stream of `seed`
    (tcx_sm100_random). Element i is stream element offset + i, so shards made at
    their global offsets concatenate to the whole tensor. The values are not NumPy's
    default_rng(seed) values (a host-only PCG64 + ziggurat stream)."""
    if dtype not in ("float32", torch.float32):
        raise ValueError("randn only supports float32")
    return _generate(0, shape, seed, offset, 0.0, 1.0, device)


def rand_uniform(shape, low: float = 0.0, high: float = 1.0, device="cuda", seed: int | None = None, *,
                 offset: int = 0) -> torch.Tensor:
    """Uniform float32 on [low, high) from the same counter-based stream (24 random
    bits per value)."""
    return _generate(1, shape, seed, offset, float(low), float(high), device)
