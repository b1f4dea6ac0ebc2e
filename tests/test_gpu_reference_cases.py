"""The reference's own device acceptance cases, run through this backend.

Each test restates a case of the reference's Python suite on the same inputs and checks
it the way that test does (NumPy expectation, tolerance, error type), plus the CPU oracle
bit for bit where the reduction order is the sequential one:
  tests/python/test_multi_axis_reductions.py:19-140 (sum/max/mean over axis selections)
  tests/python/test_int32_primitives.py:23-130 (int32 wraparound: binary, reductions)
  tests/python/test_inference_ops.py:51-100 (linear, affine rmsnorm/layernorm)
"""
import gc
import operator
import warnings

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.array(a, order="C")).cuda()  # keeps 0-d arrays 0-d


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    if a.dtype == np.float32:
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    else:
        np.testing.assert_array_equal(a, b)


def same_bits_or_nan(a, b):
    """Bit-exact except that NaNs match NaNs: a NaN that arithmetic creates (inf - inf)
    carries the platform's default pattern (0xFFC00000 from x86 SSE, 0x7FFFFFFF from
    the GPU); stored NaN payloads are checked bit for bit where they are copied."""
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and np.array_equal(np.isnan(a), np.isnan(b))
    keep = ~np.isnan(a)
    same_bits(a[keep], b[keep])


# ------------------------------------------------------ multi-axis reductions
CASES = [
    ((2, 3, 4), None), ((2, 3, 4), ()), ((2, 3, 4), (0, 2)),
    ((2, 3, 4), (2, 0)), ((2, 3, 4), (-1, 0)), ((2, 3, 4), (0, 1, 2)),
    ((2, 3, 4), (0, 1)), ((2, 3, 4), (1, 2)), ((2, 3, 4), (1,)),
    ((2, 3, 4), -1), ((1, 1, 1), (0, 2)), ((257, 2, 3), (1, 2)),
    ((2, 3, 257), (0, 2)), ((0, 2, 3), (1, 2)), ((2, 0, 3), (0, 2)),
    ((2, 0, 3), (1, 2)), ((2, 0, 3), None), ((2, 0, 3), ()),
    ((0, 2, 0), (0, 2)), ((0,), None), ((), None), ((), ()), ((), 0), ((), -1),
]


@pytest.mark.parametrize("name", ["sum", "max", "mean"])
@pytest.mark.parametrize("dtype", [np.float32, np.int32])
@pytest.mark.parametrize("shape,axis", CASES)
def test_multi_axis_numpy_parity(tcx, oracle, name, dtype, shape, axis):
    """test_multi_axis_reductions.py:31-60."""
    values = np.resize(np.array([-5, -1, 0, 2, 7], dtype=dtype), shape)
    x = dev(values)
    if dtype == np.int32 and name == "mean":
        for keepdims in (False, True):
            with pytest.raises(ValueError, match="float32"):
                getattr(tcx, name)(x, axis, keepdims=keepdims)
        return
    reference_axis = None if not shape and axis in (0, -1) else axis
    for keepdims in (False, True):
        kwargs = {"axis": reference_axis, "keepdims": keepdims}
        if name == "sum":
            kwargs["dtype"] = dtype  # int32 sums keep int32 and wrap
        try:
            with warnings.catch_warnings(), np.errstate(all="ignore"):
                warnings.simplefilter("ignore", RuntimeWarning)
                expected = getattr(np, name)(values, **kwargs)
        except ValueError:
            with pytest.raises(ValueError):
                getattr(tcx, name)(x, axis, keepdims=keepdims)
            continue
        for y in (getattr(tcx, name)(x, axis, keepdims=keepdims),
                  getattr(tcx, name)(x, axis=axis, keepdims=np.bool_(keepdims))):
            assert tuple(y.shape) == expected.shape and y.dtype == x.dtype and y.is_cuda
            assert y.data_ptr() != x.data_ptr() or x.numel() == 0
            got = host(y)
            np.testing.assert_allclose(got, expected, rtol=1e-5, atol=1e-5, equal_nan=True)
            same_bits_or_nan(got.reshape(-1), getattr(oracle, name)(values, axis).reshape(-1))
    same_bits(host(x), values)


@pytest.mark.parametrize("name", ["sum", "max", "mean"])
def test_multi_axis_default_and_sequence_protocol(tcx, name):
    """test_multi_axis_reductions.py:64-75: None, iterables and __index__ axes."""
    class Axis:
        def __index__(self):
            return 0
    x = dev(np.arange(24, dtype=np.float32).reshape(2, 3, 4))
    fn = getattr(tcx, name)
    same_bits(host(fn(x)), host(fn(x, None)))
    expected = host(fn(x, (0, 2)))
    for axes in ([Axis(), np.int32(2)], iter([2, 0]), np.array([0, 2])):
        same_bits(host(fn(x, axes)), expected)
    same_bits(host(fn(x, Axis())), host(fn(x, 0)))


@pytest.mark.parametrize("name", ["sum", "max", "mean"])
def test_multi_axis_validation_even_for_empty_inputs(tcx, name):
    """test_multi_axis_reductions.py:78-98."""
    fn = getattr(tcx, name)
    for shape in ((2, 3, 4), (2, 0, 4)):
        x = torch.empty(shape, dtype=torch.float32, device="cuda")
        for axes in (True, np.bool_(True), 0.5, "0", b"0", (0, 0), (0, -3),
                     (3,), (-4,), (0, True), (0, 2.0), (2**64,), (-(2**64),)):
            with pytest.raises(ValueError):
                fn(x, axes)
        for keepdims in (1, None, "yes", []):
            with pytest.raises(TypeError, match="keepdims"):
                fn(x, (0, 2), keepdims=keepdims)
    scalar = dev(np.array(1.0, np.float32))
    for axes in ((0,), (-1,), 1, -2):
        with pytest.raises(ValueError):
            fn(scalar, axes)
    with pytest.raises(TypeError):
        fn([1.0], None)


@pytest.mark.parametrize("name", ["sum", "max", "mean"])
def test_multi_axis_empty_selection_copies_stored_bits(tcx, name):
    """test_multi_axis_reductions.py:101-111: axis=() returns a copy of the stored
    bits (signed zero, NaN payload, subnormal, inf) that outlives the input."""
    bits = np.array([0x80000000, 0x7FC12345, 1, 0x7F800000], dtype=np.uint32)
    x = dev(bits.view(np.float32))
    y = getattr(tcx, name)(x, ())
    assert y.data_ptr() != x.data_ptr()
    del x
    gc.collect()
    np.testing.assert_array_equal(host(y).view(np.uint32), bits)


@pytest.mark.parametrize("name", ["sum", "max", "mean"])
def test_multi_axis_special_values_and_canonical_order(tcx, oracle, name):
    """test_multi_axis_reductions.py:114-131: every axis spelling equals the one-pass
    row-major reduction of the flattened tensor, signed zeros included."""
    for values in ([[0., -0.], [-0., 0.]], [[np.inf, 2], [-np.inf, 4]],
                   [[1, np.nan], [3, 4]], [[3e38, 3e38], [-3e38, -3e38]],
                   [[1e20, 1], [-1e20, 3]]):
        data = np.array(values, dtype=np.float32)
        expected = getattr(oracle, name)(data.reshape(-1), 0)
        x = dev(data)
        for axes in (None, (0, 1), (1, 0), (-1, -2)):
            actual = host(getattr(tcx, name)(x, axes))
            np.testing.assert_allclose(actual, expected, equal_nan=True)
            same_bits_or_nan(actual, expected)
            if expected == 0:
                assert np.signbit(actual) == np.signbit(expected)
    if name == "mean":
        # One sum then one division gives +inf where sequential means would give NaN.
        assert np.isposinf(host(tcx.mean(dev(np.array([[3e38, 3e38], [-3e38, -3e38]], np.float32)),
                                         (0, 1))))


def test_multi_axis_int32_wrap_and_dtype_rejection(tcx):
    """test_multi_axis_reductions.py:134-141."""
    data = np.array([[2**31 - 1, 2**31 - 1], [-2**31, -17]], dtype=np.int32)
    x = dev(data)
    for axes in (None, (), (0, 1)):
        np.testing.assert_array_equal(host(tcx.sum(x, axes)), data.sum(axis=axes, dtype=np.int32))
        np.testing.assert_array_equal(host(tcx.max(x, axes)), data.max(axis=axes))
        with pytest.raises(ValueError, match="float32"):
            tcx.mean(x, axes)


# --------------------------------------------------------------- int32 exact
EDGES = np.array([-2**31, 2**31 - 1, -16777217, 16777217, -1, 0, 1, 65537], dtype=np.int32)
SHAPES = [(), (0,), (2, 0, 3), (1,), (255,), (256,), (257,), (3, 257), (2, 3, 5)]
OPS = [("add", operator.add), ("subtract", operator.sub), ("multiply", operator.mul)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("op", OPS, ids=lambda o: o[0])
def test_int32_binary_exact_wrap(tcx, shape, op):
    """test_int32_primitives.py:44-54."""
    a, b = np.resize(EDGES, shape), np.resize(EDGES[::-1], shape)
    with np.errstate(over="ignore"):
        expected = op[1](a, b)
    x, y = dev(a), dev(b)
    out = getattr(tcx, op[0])(x, y)
    assert out.dtype == torch.int32 and tuple(out.shape) == expected.shape
    np.testing.assert_array_equal(host(out), expected)
    np.testing.assert_array_equal(host(x), a)
    np.testing.assert_array_equal(host(y), b)


@pytest.mark.parametrize("op", OPS, ids=lambda o: o[0])
@pytest.mark.parametrize("shapes", [((2, 1, 257), (3, 1)), ((257,), ()), ((), (257,)),
                                    ((2, 0, 3), (1, 3)), ((0, 3), (1, 3))])
def test_int32_broadcast_exact_wrap(tcx, op, shapes):
    """test_int32_primitives.py:80-90."""
    a, b = (np.resize(EDGES, s) for s in shapes)
    with np.errstate(over="ignore"):
        expected = op[1](a, b)
    np.testing.assert_array_equal(host(getattr(tcx, op[0])(dev(a), dev(b))), expected)


REDUCTIONS = [((2, 3, 257), 0), ((2, 3, 257), 1), ((3, 257), -1),
              ((2, 3, 257), (0, 2)), ((2, 3, 257), (2, 0)), ((3, 257), None),
              ((2, 3), ()), ((2, 0, 3), 1), ((0, 2, 3), (1, 2)),
              ((0, 2, 3), (0, 2)), ((2, 0, 3), None), ((), 0), ((), -1), ((), None)]


@pytest.mark.parametrize("shape,axes", REDUCTIONS)
@pytest.mark.parametrize("name", ["sum", "max"])
@pytest.mark.parametrize("keepdims", [False, True])
def test_int32_reductions_exact_wrap(tcx, shape, axes, name, keepdims):
    """test_int32_primitives.py:100-116."""
    a = np.resize(EDGES, shape)
    x = dev(a)
    kwargs = dict(axis=None if not shape and axes in (0, -1) else axes, keepdims=keepdims)
    if name == "sum":
        kwargs["dtype"] = np.int32
    try:
        expected = getattr(np, name)(a, **kwargs)
    except ValueError:
        with pytest.raises(ValueError, match="non-empty"):
            getattr(tcx, name)(x, axes, keepdims=keepdims)
    else:
        out = getattr(tcx, name)(x, axes, keepdims=keepdims)
        assert out.dtype == torch.int32 and tuple(out.shape) == np.shape(expected)
        np.testing.assert_array_equal(host(out), expected)
    np.testing.assert_array_equal(host(x), a)


@pytest.mark.parametrize("op", OPS, ids=lambda o: o[0])
def test_int32_random_bits_and_signed_max(tcx, op):
    """test_int32_primitives.py:119-130."""
    rng = np.random.default_rng(4401)
    a, b = (rng.integers(0, 2**32, size=(7, 1027), dtype=np.uint32).view(np.int32) for _ in range(2))
    x, y = dev(a), dev(b)
    with np.errstate(over="ignore"):
        expected = op[1](a, b)
    np.testing.assert_array_equal(host(getattr(tcx, op[0])(x, y)), expected)
    np.testing.assert_array_equal(host(tcx.sum(x, (0, 1))), a.sum(dtype=np.int32))
    np.testing.assert_array_equal(host(tcx.max(x, 1)), a.max(axis=1))
    negatives = np.array([[-2**31, -7, -16777217]], dtype=np.int32)
    np.testing.assert_array_equal(host(tcx.max(dev(negatives), 1)), negatives.max(axis=1))


# ------------------------------------------------------------ inference ops
def f32(shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


@pytest.mark.parametrize("shape,out", [((3,), 4), ((2, 3), 5), ((2, 1, 4, 3), 2),
                                       ((0, 3), 2), ((2, 0), 3), ((2, 3), 0), ((0,), 2)])
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("path", ["auto", "ffma"])
def test_linear_parity(tcx, oracle, shape, out, bias, path):
    """test_inference_ops.py:51-65: x @ w.T + b for 1-d, batched and empty inputs."""
    a, w, b = f32(shape), f32((out, shape[-1]), 4), f32((out,), 9)
    expected = a @ w.T + (b if bias else 0)
    x, weight, offset = dev(a), dev(w), dev(b)
    y = tcx.linear(x, weight, offset if bias else None, path=path)
    got = host(y)
    assert got.shape == expected.shape
    np.testing.assert_allclose(got, expected, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got, oracle.linear(a, w, b if bias else None), rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(host(x), a)
    np.testing.assert_array_equal(host(weight), w)


@pytest.mark.parametrize("shape,axis", [((2, 3, 4), -1), ((2, 3, 4), 1), ((2, 3, 4), 0),
                                        ((3,), -1), ((), 0), ((), -1), ((0, 3), 1), ((2, 0, 3), 1)])
@pytest.mark.parametrize("kind,params", [("rmsnorm", "weight"), ("layernorm", "weight"),
                                         ("layernorm", "both"), ("layernorm", "bias")])
def test_affine_norm_parity(tcx, shape, axis, kind, params):
    """test_inference_ops.py:68-100: normalized, then * weight, then + bias, along
    any axis, for scalars and empty tensors too."""
    a = f32(shape)
    pshape = (shape[axis],) if shape else ()
    w, b = f32(pshape, 5), f32(pshape, 6)
    kwargs = {}
    if params in ("weight", "both"):
        kwargs["weight"] = dev(w)
    if params in ("bias", "both"):
        kwargs["bias"] = dev(b)
    with np.errstate(all="ignore"):
        if a.size or not shape:
            red = axis if shape else None
            base = a if kind == "rmsnorm" else a - np.mean(a, axis=red, keepdims=True)
            expected = base / np.sqrt(np.mean(base * base, axis=red, keepdims=True) + np.float32(1e-5))
        else:
            expected = np.empty(shape, np.float32)
        pview = [1] * len(shape)
        if shape:
            pview[axis] = shape[axis]
        if "weight" in kwargs:
            expected = expected * w.reshape(pview)
        if "bias" in kwargs:
            expected = expected + b.reshape(pview)
    x = dev(a)
    got = host(getattr(tcx, kind)(x, axis, **kwargs))
    assert got.shape == np.shape(expected)
    np.testing.assert_allclose(got, expected, rtol=1e-5, atol=1e-5, equal_nan=True)
    # weight=None is the unweighted op
    same_bits(host(getattr(tcx, kind)(x, axis, weight=None)), host(getattr(tcx, kind)(x, axis)))


# ------------------------------------------------------------------ attention
def numpy_attention(q, k, v, mask=None, causal=False, scale=None):
    """Float64-free NumPy statement of the kAttention contract (scale * q·kᵀ, then a
    bool mask selects, a float mask adds and -inf in it selects, causal keeps
    key <= query, fully masked rows give zeros)."""
    batch = np.broadcast_shapes(q.shape[:-2], k.shape[:-2], v.shape[:-2])
    lq, lk = q.shape[-2], k.shape[-2]
    s = np.float32(1 / np.sqrt(q.shape[-1]) if scale is None else scale)
    logits = np.broadcast_to(np.matmul(q, np.swapaxes(k, -1, -2)), batch + (lq, lk)) * s
    keep = np.ones(batch + (lq, lk), bool)
    if causal:
        keep = keep & np.tri(lq, lk, dtype=bool)
    if mask is not None:
        if mask.dtype == np.bool_:
            keep = keep & mask
        else:
            keep = keep & (mask != -np.inf)
            logits = logits + mask
    logits = np.where(keep, logits, -np.inf).astype(np.float32)
    if lk == 0:
        return np.zeros(batch + (lq, v.shape[-1]), np.float32)
    with np.errstate(all="ignore"):
        top = logits.max(axis=-1, keepdims=True)
        e = np.exp(logits - top)
        p = np.where(top == -np.inf, np.float32(0), e / e.sum(axis=-1, keepdims=True))
        return (p @ v).astype(np.float32)


def attn_check(got, expected):
    assert got.shape == expected.shape, (got.shape, expected.shape)
    np.testing.assert_allclose(got, expected, rtol=2e-4, atol=2e-5, equal_nan=True)


def gauss(shape, seed=31):
    return np.random.default_rng(seed).normal(size=shape).astype(np.float32)


ATTN_SHAPES = [((3, 4), (5, 4), (5, 2)), ((2, 3, 4), (2, 5, 4), (2, 5, 6)),
               ((2, 1, 3, 4), (1, 3, 5, 4), (2, 3, 5, 2)), ((3, 4), (5, 4), (2, 1, 5, 2)),
               ((0, 4), (5, 4), (5, 2)), ((3, 4), (0, 4), (0, 2)),
               ((0, 3, 4), (1, 5, 4), (1, 5, 2)), ((3, 4), (5, 4), (5, 0))]


def attn_mask(kind, mshape):
    rng = np.random.default_rng(41)
    if kind == "bool":
        m = rng.random(mshape) > 0.4
        if m.shape[0]:
            m[0] = False
        return m
    if kind == "additive":
        m = gauss(mshape)
        m[rng.random(mshape) < 0.3] = -np.inf
        if m.shape[0]:
            m[0] = -np.inf
        return m
    if kind == "scalar_false":
        return np.array(False)
    return None


@pytest.mark.parametrize("shapes", ATTN_SHAPES)
@pytest.mark.parametrize("mask_kind", ["none", "bool", "additive", "scalar_false"])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_parity(tcx, oracle, shapes, mask_kind, causal):
    """test_inference_ops.py:136-155: broadcast batches, empty extents, every mask
    kind, causal or not; the oracle is the reference composite restated."""
    q, k, v = [gauss(s, i + 10) for i, s in enumerate(shapes)]
    mask = attn_mask(mask_kind, (q.shape[-2], k.shape[-2]))
    got = host(tcx.attention(dev(q), dev(k), dev(v), None if mask is None else dev(mask), is_causal=causal))
    attn_check(got, numpy_attention(q, k, v, mask, causal))
    attn_check(got, oracle.attention(q, k, v, mask, causal))


@pytest.mark.parametrize("scale", [0, -0.5, 2, np.float32(0.3)])
def test_attention_scale_and_batched_mask(tcx, scale):
    """test_inference_ops.py:158-164."""
    q, k, v = gauss((2, 3, 4)), gauss((5, 4), 2), gauss((5, 3), 3)
    mask = np.random.default_rng(4).random((2, 1, 5)) > 0.3
    got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask), scale=scale))
    attn_check(got, numpy_attention(q, k, v, mask, scale=scale))


def test_attention_causality(tcx):
    """test_inference_ops.py:167-174: causal rows never see later keys or values."""
    q, k, v = gauss((5, 4)), gauss((5, 4), 2), gauss((5, 3), 3)
    before = host(tcx.attention(dev(q), dev(k), dev(v), is_causal=True))
    k[3:] += 100
    v[3:] -= 500
    after = host(tcx.attention(dev(q), dev(k), dev(v), is_causal=True))
    np.testing.assert_array_equal(before[:3], after[:3])


@pytest.mark.parametrize("exceptional", [np.nan, np.inf, -np.inf])
@pytest.mark.parametrize("masked", [False, True])
def test_attention_nonfinite_scores(tcx, oracle, exceptional, masked):
    """test_inference_ops.py:177-184: inf/NaN keys, masked or not."""
    q, k, v = np.ones((1, 2), np.float32), np.ones((2, 2), np.float32), gauss((2, 3))
    k[0] = exceptional
    mask = np.array([[not masked, True]])
    got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask)))
    with np.errstate(all="ignore"):
        attn_check(got, numpy_attention(q, k, v, mask))
        attn_check(got, oracle.attention(q, k, v, mask))


@pytest.mark.parametrize("scale", [np.nan, np.inf, -np.inf, 1e300, 1e-300, 10**400])
def test_attention_invalid_scale_even_empty(tcx, scale):
    """test_inference_ops.py:187-190."""
    q, k, v = (torch.zeros(s, device="cuda") for s in ((0, 2), (3, 2), (3, 1)))
    with pytest.raises(ValueError):
        tcx.attention(q, k, v, scale=scale)


@pytest.mark.parametrize("scale", [True, "2", 1j, [1]])
def test_attention_invalid_scale_type(tcx, scale):
    """test_inference_ops.py:193-196."""
    x = torch.ones((2, 2), device="cuda")
    with pytest.raises(TypeError):
        tcx.attention(x, x, x, scale=scale)


@pytest.mark.parametrize("case", ["rank", "features", "zero_features", "sequence", "batch", "mask_int",
                                  "mask_shape", "mask_rank", "int"])
def test_attention_invalid_contract(tcx, case):
    """test_inference_ops.py:213-238, the attention rows."""
    def t(shape, dtype=torch.float32):
        return torch.zeros(shape, dtype=dtype, device="cuda")
    calls = {
        "rank": lambda: tcx.attention(t((3,)), t((2, 3)), t((2, 3))),
        "features": lambda: tcx.attention(t((0, 3)), t((2, 4)), t((2, 3))),
        "zero_features": lambda: tcx.attention(t((0, 0)), t((2, 0)), t((2, 3))),
        "sequence": lambda: tcx.attention(t((0, 3)), t((2, 3)), t((3, 3))),
        "batch": lambda: tcx.attention(t((2, 0, 3)), t((3, 2, 3)), t((3, 2, 3))),
        "mask_int": lambda: tcx.attention(t((0, 3)), t((2, 3)), t((2, 3)), t((0, 2), torch.int32)),
        "mask_shape": lambda: tcx.attention(t((0, 3)), t((2, 3)), t((2, 3)), t((0, 3), torch.bool)),
        "mask_rank": lambda: tcx.attention(t((0, 3)), t((2, 3)), t((2, 3)), t((1, 0, 2), torch.bool)),
        "int": lambda: tcx.attention(t((0, 3), torch.int32), t((2, 3)), t((2, 3))),
    }
    with pytest.raises(ValueError):
        calls[case]()


@pytest.mark.parametrize("scale", [1e-39, -1e-39, 1e-40, -1e-40])
def test_attention_subnormal_scale(tcx, scale):
    """test_inference_ops.py:283-287: subnormal scales survive the float32 narrowing."""
    q, k, v = np.array([[1]], np.float32), np.array([[0], [1e38]], np.float32), np.array([[0], [1]], np.float32)
    got = host(tcx.attention(dev(q), dev(k), dev(v), scale=scale))
    attn_check(got, numpy_attention(q, k, v, scale=scale))


def test_attention_huge_empty_batch(tcx):
    """test_inference_ops.py:290-294, with 2**40 for the reference's 2**62 (a torch
    tensor's strides overflow at 2**62 even when it is empty)."""
    q = torch.empty((0, 2**40, 4, 0, 2), device="cuda")
    v = torch.empty((0, 2**40, 4, 0, 3), device="cuda")
    out = tcx.attention(q, q, v)
    assert tuple(out.shape) == tuple(v.shape)


def test_attention_high_rank_metadata(tcx):
    """test_inference_ops.py:297-302: 17 batch axes."""
    shape = (1,) * 17
    q, k, v = gauss(shape + (3, 4)), gauss(shape + (2, 4), 2), gauss(shape + (2, 3), 3)
    attn_check(host(tcx.attention(dev(q), dev(k), dev(v))), numpy_attention(q, k, v))


@pytest.mark.parametrize("lq,lk,d,dv", [(64, 300, 32, 16), (256, 1024, 64, 64), (128, 2048, 128, 128),
                                        (200, 4096, 64, 80), (64, 8192, 64, 64), (16, 20000, 32, 32)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_sizes_through_every_softmax_width(tcx, oracle, lq, lk, d, dv, causal):
    """Sizes that reach the tcgen05 GEMMs and each register / streaming softmax shape,
    against the restated reference composite."""
    q, k, v = gauss((2, lq, d), 1), gauss((2, lk, d), 2), gauss((2, lk, dv), 3)
    mask = np.random.default_rng(5).random((lq, lk)) > 0.2
    got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask), is_causal=causal))
    attn_check(got, oracle.attention(q, k, v, mask, causal))


@pytest.mark.parametrize("shape,sshape,mshape,kind", [
    ((4, 7), (4, 7), None, None), ((2, 3, 130), (3, 130), (2, 1, 130), "bool"),
    ((2, 5, 600), (2, 5, 600), (600,), "float"), ((3, 2100), (1, 2100), (3, 1), "bool"),
    ((2, 9000), (2, 9000), (2, 9000), "float"), ((2, 3, 4), (2, 3, 1), (3, 4), "float")])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_softmax_primitive(tcx, oracle, shape, sshape, mshape, kind, causal):
    """kAttentionSoftmax with broadcast scores and masks (core/inference.cpp:56-83)."""
    scores = gauss(sshape, 8) * 4
    mask = None
    if kind == "bool":
        mask = np.random.default_rng(9).random(mshape) > 0.3
    elif kind == "float":
        mask = gauss(mshape, 10)
        mask[np.random.default_rng(11).random(mshape) < 0.2] = -np.inf
    got = host(tcx.attention_softmax(dev(scores), shape, None if mask is None else dev(mask), scale=0.7,
                                     is_causal=causal))
    want = oracle.attention_softmax(scores, shape, mask, causal, 0.7)
    assert got.shape == want.shape
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7, equal_nan=True)


@pytest.mark.parametrize("lq,lk,d,dv", [(128, 128, 32, 32), (200, 300, 64, 64), (1, 5, 32, 64), (300, 77, 96, 32),
                                        (256, 1000, 128, 128), (130, 2049, 64, 96), (2048, 2048, 128, 128)])
@pytest.mark.parametrize("causal", [False, True])
def test_fused_attention(tcx, oracle, lq, lk, d, dv, causal):
    """No mask and feature sizes that are multiples of 32: the fused tcgen05 kernel
    (scores and probabilities in TMEM), against the restated reference composite."""
    q, k, v = gauss((2, lq, d), 1), gauss((2, lk, d), 2), gauss((2, lk, dv), 3)
    got = host(tcx.attention(dev(q), dev(k), dev(v), is_causal=causal))
    if lq * lk > 500_000:  # the CPU composite is slow here: check the first rows only
        attn_check(got[:, :64], oracle.attention(q[:, :64], k, v, None, causal))
    else:
        attn_check(got, oracle.attention(q, k, v, None, causal))


@pytest.mark.parametrize("causal", [False, True])
def test_fused_attention_key_range_units(tcx, oracle, causal):
    """Fewer 256-query items than SM pairs (2 heads x 8 query tiles): the CTA-pair kernel
    cuts each item's key blocks into units of 4 (the last query tiles into up to eight),
    leaves each unit's unnormalized rows with their maxima and sums, and a combining
    kernel merges them. Every row against the reference composite; a second call is bit
    identical."""
    q, k, v = gauss((2, 2048, 128), 23), gauss((2, 2048, 128), 24), gauss((2, 2048, 128), 25)
    qd, kd, vd = dev(q), dev(k), dev(v)
    got = host(tcx.attention(qd, kd, vd, is_causal=causal))
    attn_check(got, oracle.attention(q, k, v, None, causal))
    np.testing.assert_array_equal(host(tcx.attention(qd, kd, vd, is_causal=causal)), got)


@pytest.mark.parametrize("scale", [None, 0.0, -0.3, 3.0])
def test_fused_attention_broadcast_and_scale(tcx, oracle, scale):
    q, k, v = gauss((3, 2, 100, 64), 4), gauss((1, 2, 260, 64), 5), gauss((3, 1, 260, 32), 6)
    got = host(tcx.attention(dev(q), dev(k), dev(v), scale=scale, is_causal=True))
    attn_check(got, oracle.attention(q, k, v, None, True, scale))


@pytest.mark.parametrize("where", ["q", "k", "v"])
@pytest.mark.parametrize("value", [np.inf, -np.inf, np.nan])
def test_fused_attention_nonfinite_inputs(tcx, oracle, where, value):
    """inf / NaN anywhere sends the work to the IEEE row kernel, which follows the
    reference composite (masked keys included in P·V, as its dense product does)."""
    q, k, v = gauss((1, 70, 32), 7), gauss((1, 90, 32), 8), gauss((1, 90, 32), 9)
    {"q": q, "k": k, "v": v}[where][0, 3, 5] = value
    for causal in (False, True):
        got = host(tcx.attention(dev(q), dev(k), dev(v), is_causal=causal))
        with np.errstate(all="ignore"):
            attn_check(got, oracle.attention(q, k, v, None, causal))


@pytest.mark.parametrize("where,index", [("q", (0, 150, 5)), ("k", (1, 350, 7)), ("v", (0, 399, 63)),
                                         ("v", (1, 0, 0))])
@pytest.mark.parametrize("value", [np.inf, np.nan])
@pytest.mark.parametrize("lq", [300, 200])
def test_fused_attention_pair_nonfinite_inputs(tcx, oracle, where, index, value, lq):
    """The CTA-pair kernel (over 128 queries, Dv 64 or 128) reads q, k, v in place and
    checks them for inf / NaN on the way; a hit anywhere, even at keys no query reaches
    causally (with 200 queries, k and v rows 256-399 are never loaded and are scanned
    apart), hands the call to the IEEE row kernel."""
    q, k, v = gauss((2, lq, 64), 17), gauss((2, 400, 64), 18), gauss((2, 400, 64), 19)
    {"q": q, "k": k, "v": v}[where][index] = value
    for causal in (False, True):
        got = host(tcx.attention(dev(q), dev(k), dev(v), is_causal=causal))
        with np.errstate(all="ignore"):
            attn_check(got, oracle.attention(q, k, v, None, causal))


def test_fused_attention_pair_broadcast(tcx, oracle):
    """Broadcast batch axes through the pair kernel's in-place operand maps: k shared
    over the first batch axis, v over the second."""
    q, k, v = gauss((3, 2, 300, 64), 20), gauss((1, 2, 260, 64), 21), gauss((3, 1, 260, 128), 22)
    for causal in (False, True):
        got = host(tcx.attention(dev(q), dev(k), dev(v), scale=0.4, is_causal=causal))
        attn_check(got, oracle.attention(q, k, v, None, causal, 0.4))


FUSED_MASKS = [
    # (mask shape relative to [batch=2, L, S], kind): full, broadcast over batch or queries,
    # constant along keys (key stride 0), a scalar
    ("LS", "bool"), ("LS", "additive"), ("B1S", "bool"), ("B1S", "additive"), ("1S", "additive"),
    ("L1", "bool"), ("L1", "additive"), ("scalar", "bool"), ("BLS", "additive")]


def fused_mask(kind, form, b, lq, lk, seed=43):
    shape = {"LS": (lq, lk), "B1S": (b, 1, lk), "1S": (1, lk), "L1": (lq, 1), "scalar": (), "BLS": (b, lq, lk)}[form]
    rng = np.random.default_rng(seed)
    if kind == "bool":
        m = rng.random(shape) > 0.35
        if form == "scalar":
            return np.array(True)
        if form in ("LS", "L1"):
            m[min(2, lq - 1)] = False  # a fully masked row: zeros
        return m
    m = rng.normal(size=shape).astype(np.float32)
    m[rng.random(shape) < 0.3] = -np.inf
    if form in ("LS", "L1", "BLS"):
        m[..., min(2, lq - 1), :] = -np.inf
    return m


@pytest.mark.parametrize("lq,lk,d,dv", [(130, 200, 32, 32), (64, 257, 64, 96), (200, 128, 128, 64)])
@pytest.mark.parametrize("form,kind", FUSED_MASKS)
@pytest.mark.parametrize("causal", [False, True])
def test_fused_attention_masked(tcx, oracle, lq, lk, d, dv, form, kind, causal):
    """Masks inside the fused tcgen05 kernel (feature sizes that are multiples of 32):
    every broadcast form of a bool or float mask, -inf entries, rows with no unmasked
    key (zeros), keys that do not fill the last 64-key block, causal or not; against
    the restated reference composite and NumPy."""
    q, k, v = gauss((2, lq, d), 21), gauss((2, lk, d), 22), gauss((2, lk, dv), 23)
    mask = fused_mask(kind, form, 2, lq, lk)
    got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask), is_causal=causal))
    attn_check(got, oracle.attention(q, k, v, mask, causal))
    attn_check(got, numpy_attention(q, k, v, mask, causal))


def test_fused_attention_masked_unaligned_rows(tcx, oracle):
    """Mask rows that do not start on a 16-byte boundary (odd key count) take the
    element-wise mask loads."""
    q, k, v = gauss((1, 70, 32), 24), gauss((1, 131, 32), 25), gauss((1, 131, 32), 26)
    for kind in ("bool", "additive"):
        mask = fused_mask(kind, "LS", 1, 70, 131, seed=44)
        got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask)))
        attn_check(got, oracle.attention(q, k, v, mask, False))


@pytest.mark.parametrize("value", [np.nan, np.inf])
def test_fused_attention_mask_nonfinite(tcx, oracle, value):
    """NaN or +inf in a float mask sends the call to the IEEE row kernel: the reference
    composite's NaN rows (a NaN score, or +inf - +inf)."""
    q, k, v = gauss((1, 70, 32), 27), gauss((1, 90, 32), 28), gauss((1, 90, 32), 29)
    mask = fused_mask("additive", "LS", 1, 70, 90, seed=45)
    mask[5, 7] = value
    for causal in (False, True):
        got = host(tcx.attention(dev(q), dev(k), dev(v), dev(mask), is_causal=causal))
        with np.errstate(all="ignore"):
            attn_check(got, oracle.attention(q, k, v, mask, causal))


# ------------------------------------------------------------ min / argmax / clip
MIN_CASES = [((), None), ((), 0), ((), -1), ((), ()), ((2, 3, 4), None), ((2, 3, 4), 0), ((2, 3, 4), -1),
             ((2, 3, 4), (0, 2)), ((2, 3, 4), (-1, 0)), ((2, 3, 4), ()), ((0, 3), 1), ((2, 0, 3), 0)]


@pytest.mark.parametrize("dtype", [np.float32, np.int32])
@pytest.mark.parametrize("shape,axis", MIN_CASES)
@pytest.mark.parametrize("keepdims", [False, True])
def test_min_parity(tcx, dtype, shape, axis, keepdims):
    """test_math_ops.py:62-72."""
    a = np.random.default_rng(42).integers(-500, 500, shape).astype(dtype)
    x = dev(a)
    try:
        expected = np.min(a, axis=axis, keepdims=keepdims)
    except ValueError:
        with pytest.raises(ValueError):
            tcx.min(x, axis, keepdims=keepdims)
        return
    got = host(tcx.min(x, axis, keepdims=keepdims))
    assert got.shape == np.shape(expected)
    np.testing.assert_array_equal(got, expected)


ARGMAX_CASES = [((), None), ((), 0), ((), -1), ((2, 3, 4), None), ((2, 3, 4), 0), ((2, 3, 4), 1),
                ((2, 3, 4), -1), ((0, 3), 1), ((2, 0, 3), 0)]


@pytest.mark.parametrize("dtype", [np.float32, np.int32])
@pytest.mark.parametrize("shape,axis", ARGMAX_CASES)
@pytest.mark.parametrize("keepdims", [False, True])
def test_argmax_parity(tcx, dtype, shape, axis, keepdims):
    """test_math_ops.py:75-83: first maximum, int32 indices."""
    a = np.random.default_rng(73).integers(-3, 4, shape).astype(dtype)
    x = dev(a)
    try:
        expected = np.asarray(np.argmax(a, axis=axis, keepdims=keepdims), dtype=np.int32)
    except ValueError:
        with pytest.raises(ValueError):
            tcx.argmax(x, axis, keepdims=keepdims)
        return
    got = host(tcx.argmax(x, axis, keepdims=keepdims))
    assert got.dtype == np.int32 and got.shape == expected.shape
    np.testing.assert_array_equal(got, expected)


@pytest.mark.parametrize("axis", [None, 0, 1, -1])
def test_min_argmax_ieee_ties(tcx, axis):
    """test_math_ops.py:86-91: NaN wins, both zeros equal, the lowest index on ties."""
    a = np.array([[0., -0., 1e-40, -1e-40, np.inf], [np.nan, 2., np.nan, -np.inf, 2.]], np.float32)
    x = dev(a)
    np.testing.assert_array_equal(host(tcx.min(x, axis)), np.min(a, axis=axis))
    np.testing.assert_array_equal(host(tcx.argmax(x, axis)), np.asarray(np.argmax(a, axis=axis), np.int32))


def test_min_signed_zero_first_value(tcx):
    """test_math_ops.py:226-233: among equal zeros the first one's bits are returned."""
    bits = np.array([[0, 0x80000000], [0x80000000, 0]], np.uint32)
    x = dev(bits.view(np.float32))
    np.testing.assert_array_equal(host(tcx.min(x, 1)).view(np.uint32), bits[:, 0])
    np.testing.assert_array_equal(host(tcx.argmax(x, 1)), [0, 0])


@pytest.mark.parametrize("dtype", [np.float32, np.int32])
@pytest.mark.parametrize("bounds", [(-2, 3), (None, 3), (-2, None), (4, -4), (0, 0)])
@pytest.mark.parametrize("shape", [(), (0,), (2, 3, 4)])
def test_clip_scalar_parity(tcx, dtype, bounds, shape):
    """test_math_ops.py:94-102."""
    a = np.random.default_rng(75).integers(-10, 10, shape).astype(dtype)
    got = host(tcx.clip(dev(a), *bounds))
    expected = np.asarray(np.clip(a, *bounds), dtype=dtype)
    assert got.shape == expected.shape
    np.testing.assert_array_equal(got, expected)


@pytest.mark.parametrize("dtype", [np.float32, np.int32])
def test_clip_broadcast_bounds(tcx, dtype):
    """test_math_ops.py:105-113: bounds broadcast the output beyond the input's shape."""
    a = np.array([[[-4], [1], [9]]], dtype=dtype)
    lo = np.array([[-1, 2, 7, 8]], dtype=dtype)
    hi = np.array([[[3]], [[10]]], dtype=dtype)
    got = host(tcx.clip(dev(a), dev(lo), dev(hi)))
    np.testing.assert_array_equal(got, np.clip(a, lo, hi))


def test_clip_ieee(tcx):
    """test_math_ops.py:116-122: NaN in the input or a bound propagates; signed zeros and
    subnormals keep their bits."""
    a = np.array([np.nan, -0., 0., 1e-40, -1e-40, np.inf, -np.inf, 1., 2.], np.float32)
    lo = np.array([-1., 0., -0., -2e-40, -2e-40, -1., -1., np.nan, -1.], np.float32)
    hi = np.array([1., 0., -0., 2e-40, 2e-40, 1., 1., 2., np.nan], np.float32)
    got = host(tcx.clip(dev(a), dev(lo), dev(hi)))
    np.testing.assert_array_equal(got, np.clip(a, lo, hi))
    np.testing.assert_array_equal(got[1:7].view(np.uint32), np.clip(a, lo, hi)[1:7].view(np.uint32))


def test_clip_empty_broadcast(tcx):
    """test_math_ops.py:237-241: an empty input broadcast against a bound."""
    for dtype in (np.float32, np.int32):
        x = dev(np.empty((0, 2, 1), dtype=dtype))
        got = host(tcx.clip(x, dev(np.zeros((1, 3), dtype=dtype)), 4))
        assert got.shape == (0, 2, 3) and got.dtype == dtype


def test_math_errors(tcx):
    """test_math_ops.py:191-223, the min / argmax / clip rows."""
    x = dev(np.array([[1., 2.]], np.float32))
    for shape in [(2, 0), (0, 0)]:
        empty = torch.empty(shape, device="cuda")
        for name in ("min", "argmax"):
            with pytest.raises(ValueError):
                getattr(tcx, name)(empty, axis=1)
    for axis in [2, -3, (0, 1), True, 1.5]:
        with pytest.raises((ValueError, TypeError)):
            tcx.argmax(x, axis)
    with pytest.raises(ValueError):
        tcx.clip(x)
    with pytest.raises(ValueError):
        tcx.clip(x, dev(np.array(1, np.int32)), 2)
    with pytest.raises(ValueError):
        tcx.clip(x, torch.ones((3,), device="cuda"), 2)
    for name in ("min", "argmax"):
        with pytest.raises(TypeError):
            getattr(tcx, name)(x, keepdims=1)
    with pytest.raises(ValueError):
        tcx.min(x, (0, 0))


def test_concurrent_inference_chain(tcx, oracle):
    """test_cuda_primitives.py:90-101: the same chain from four threads at once
    (softmax(matmul(gelu(layernorm(matmul(x, w1))), w2))), each result checked."""
    from concurrent.futures import ThreadPoolExecutor
    rng = np.random.default_rng(19)
    x = rng.normal(size=(7, 17)).astype(np.float32)
    w1 = rng.normal(size=(17, 31)).astype(np.float32)
    w2 = rng.normal(size=(31, 5)).astype(np.float32)
    expected = oracle.softmax(oracle.matmul(oracle.gelu(oracle.layernorm(oracle.matmul(x, w1), -1)), w2), -1)
    gx, g1, g2 = dev(x), dev(w1), dev(w2)

    def forward():
        torch.cuda.set_device(0)
        y = tcx.softmax(tcx.matmul(tcx.gelu(tcx.layernorm(tcx.matmul(gx, g1), -1)), g2), -1)
        torch.cuda.current_stream().synchronize()
        return y.cpu().numpy()

    with ThreadPoolExecutor(max_workers=4) as pool:
        results = [f.result() for f in [pool.submit(forward) for _ in range(12)]]
    for r in results:
        np.testing.assert_allclose(r, expected, rtol=1e-4, atol=1e-5)
