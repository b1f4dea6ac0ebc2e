"""GPU parity of row softmax / rmsnorm / layernorm (+affine) and the elementwise
kernels against the CPU oracle. Tolerances are the reference's own
(python/tensorcx/testing.py:17-21): 1e-5 rtol/atol for row ops, 1e-6 for
elementwise; add/subtract/multiply/divide and clip/ReLU are bit-exact."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROW_OPS = ["softmax", "rmsnorm", "layernorm"]


def dev(a):
    return torch.from_numpy(np.array(a, order="C")).cuda()  # keeps 0-d arrays 0-d


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(a, b, tol):
    np.testing.assert_allclose(a, b, rtol=tol, atol=tol, equal_nan=True)


def exact_row_op(op, x, axis, eps=1e-5):
    """float64 evaluation of the reference formulas (cpu_backend.cpp:125-240)."""
    x = x.astype(np.float64)
    with np.errstate(all="ignore"):
        if op == "softmax":
            e = np.exp(x - np.max(x, axis=axis, keepdims=True))
            return e / np.sum(e, axis=axis, keepdims=True)
        if op == "rmsnorm":
            return x / np.sqrt(np.mean(x * x, axis=axis, keepdims=True) + np.float32(eps))
        mean = np.mean(x, axis=axis, keepdims=True)
        return (x - mean) / np.sqrt(np.mean((x - mean) ** 2, axis=axis, keepdims=True) + np.float32(eps))


def row_close(got, cpu, exact, tol=1e-5):
    """Within the reference tolerance of the CPU result, or (elementwise) at least as
    close to the float64 result as the CPU's own float32 result is. The CPU adds the
    softmax denominator / norm statistics left to right in float32, so for wide rows
    its own error can exceed 1e-5 (terms below half an ulp of the running sum are
    dropped); a tree-ordered sum on the GPU is closer to exact there."""
    got, cpu, exact = (np.asarray(v, np.float64) for v in (got, cpu, exact))
    nan_ok = np.isnan(got) == np.isnan(cpu)
    assert nan_ok.all(), "NaN placement differs"
    fin = ~np.isnan(cpu)
    near = np.abs(got - cpu) <= tol + tol * np.abs(cpu)
    better = np.abs(got - exact) <= np.abs(cpu - exact) + 1e-7 * np.abs(exact)
    bad = fin & ~(near | better)
    assert not bad.any(), (got[bad][:5], cpu[bad][:5], exact[bad][:5])


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("width", [1, 2, 7, 33, 255, 256, 257, 1023, 1024, 1025, 2048, 2049, 4095, 4096, 4097,
                                   6000, 8192, 8193, 12000, 16384, 16385, 16392, 20004, 32768, 40000])
def test_row_ops_widths(tcx, oracle, op, width):
    rows = max(1, min(64, (1 << 20) // width))
    x = (np.random.default_rng(width).normal(size=(rows, width)) * 3).astype(np.float32)
    row_close(host(getattr(tcx, op)(dev(x), axis=-1)), getattr(oracle, op)(x, -1), exact_row_op(op, x, -1))


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("shape,axis", [((), 0), ((1,), 0), ((7,), -1), ((2, 3, 5), 0), ((2, 3, 5), 1),
                                        ((2, 0, 3), -1), ((0, 2, 3), 1), ((64, 50, 3), 1)])
def test_row_ops_axes_and_empty(tcx, oracle, op, shape, axis):
    x = np.random.default_rng(11).normal(size=shape).astype(np.float32)
    close(host(getattr(tcx, op)(dev(x), axis=axis)), getattr(oracle, op)(x, axis), 1e-5)


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("row", [[0., -0., 1e-38, -1e-38], [1., np.nan, 2., 3.], [np.inf, 1., 2., -np.inf],
                                 [1e20] * 4])
def test_row_special_values(tcx, oracle, op, row):
    a = np.array([row, row], dtype=np.float32).T.copy()
    close(host(getattr(tcx, op)(dev(a), axis=0)), getattr(oracle, op)(a, 0), 1e-5)
    b = np.array([row, row], dtype=np.float32)
    close(host(getattr(tcx, op)(dev(b), axis=1)), getattr(oracle, op)(b, 1), 1e-5)


@pytest.mark.parametrize("op", ["rmsnorm", "layernorm"])
@pytest.mark.parametrize("eps", [0.0, 1e-45, 1e-5, 1e30])
@pytest.mark.parametrize("value", [0.0, 0.3, 1e38])
@pytest.mark.parametrize("width", [33, 257, 4096, 16384, 32768])
def test_constant_rows(tcx, oracle, op, eps, value, width):
    a = np.full((3, width), value, dtype=np.float32)
    row_close(host(getattr(tcx, op)(dev(a), axis=-1, eps=eps)), getattr(oracle, op)(a, -1, eps),
              exact_row_op(op, a, -1, eps))


@pytest.mark.parametrize("op", ROW_OPS)
@pytest.mark.parametrize("width", [12000, 16384, 30000, 32768])
def test_mixed_constant_and_random_rows(tcx, oracle, op, width):
    """Rows that take different branches inside one launch (a constant layernorm row
    skips the variance exchange of the cluster kernels), interleaved with NaN rows."""
    rng = np.random.default_rng(width)
    x = (rng.normal(size=(9, width)) * 3).astype(np.float32)
    x[1] = 0.25
    x[4] = -7.0
    x[6, width // 2] = np.nan
    row_close(host(getattr(tcx, op)(dev(x), axis=-1)), getattr(oracle, op)(x, -1), exact_row_op(op, x, -1))


@pytest.mark.parametrize("op", ["rmsnorm", "layernorm"])
@pytest.mark.parametrize("eps", [-1, np.nan, np.inf, 1e100, 1e-100])
def test_bad_epsilon(tcx, op, eps):
    with pytest.raises(ValueError, match="epsilon"):
        getattr(tcx, op)(dev(np.ones((2, 3), np.float32)), axis=-1, eps=eps)


@pytest.mark.parametrize("width,axis", [(4096, -1), (300, -1), (64, 0), (6000, -1), (12000, -1), (20000, -1),
                                        (40000, -1)])
def test_affine_norms(tcx, oracle, width, axis):
    rng = np.random.default_rng(width)
    x = (rng.normal(size=(16, width)) * 3).astype(np.float32)
    n = x.shape[axis]
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    b = (rng.normal(size=n) * 0.1).astype(np.float32)
    close(host(tcx.layernorm(dev(x), axis=axis, eps=1e-5, weight=dev(w), bias=dev(b))),
          oracle.layernorm(x, axis, 1e-5, w, b), 1e-5)
    close(host(tcx.rmsnorm(dev(x), axis=axis, eps=1e-5, weight=dev(w))), oracle.rmsnorm(x, axis, 1e-5, w), 1e-5)


@pytest.mark.parametrize("op", ["exp", "gelu", "silu"])
@pytest.mark.parametrize("n", [0, 1, 257, 6, 1 << 20])
def test_unary(tcx, oracle, op, n):
    a = np.linspace(-8, 8, num=n, dtype=np.float32)
    close(host(getattr(tcx, op)(dev(a))), getattr(oracle, op)(a), 1e-6)


@pytest.mark.parametrize("op", ["exp", "gelu", "silu"])
def test_unary_special(tcx, oracle, op):
    a = np.array([0., -0., np.inf, -np.inf, np.nan, 100, -100, 1e-38], dtype=np.float32)
    close(host(getattr(tcx, op)(dev(a))), getattr(oracle, op)(a), 1e-6)


@pytest.mark.parametrize("op", ["add", "subtract", "multiply", "divide"])
@pytest.mark.parametrize("shapes", [((4, 1, 6), (3, 1)), ((1000, 37), (37,)), ((5,), (5,)), ((), (3,)),
                                    ((2, 3, 4, 5), (3, 1, 5)), ((0, 3), (3,))])
def test_binary_bit_exact(tcx, oracle, op, shapes):
    rng = np.random.default_rng(3)
    a, b = [rng.normal(size=s).astype(np.float32) for s in shapes]
    got = host(getattr(tcx, op)(dev(a), dev(b)))
    np.testing.assert_array_equal(got.view(np.uint32), getattr(oracle, op)(a, b).view(np.uint32))


def test_binary_int32_wrap(tcx, oracle):
    a = np.array([2**31 - 1, -2**31, 5, 7], np.int32)
    b = np.array([1, -1, -9, 3], np.int32)
    for op in ("add", "subtract", "multiply"):
        np.testing.assert_array_equal(host(getattr(tcx, op)(dev(a), dev(b))), getattr(oracle, op)(a, b))
    with pytest.raises(ValueError, match="float32"):
        tcx.divide(dev(a), dev(b))


@pytest.mark.parametrize("dtype", ["float32", "int32"])
@pytest.mark.parametrize("bounds", [(-2, 3), (None, 3), (-2, None), (4, -4), (0, 0)])
@pytest.mark.parametrize("shape", [(), (0,), (2, 3, 4)])
def test_clip(tcx, oracle, dtype, bounds, shape):
    a = np.random.default_rng(75).integers(-10, 10, shape).astype(dtype)
    got = host(tcx.clip(dev(a), *bounds))
    np.testing.assert_array_equal(got, oracle.clip(a, *bounds))


def test_relu_special(tcx, oracle):
    a = np.array([0., -0., np.inf, -np.inf, np.nan, 3.5, -2.0, 1e-40, -1e-40], np.float32)
    np.testing.assert_array_equal(host(tcx.relu(dev(a))).view(np.uint32), oracle.relu(a).view(np.uint32))


@pytest.mark.parametrize("act", ["none", "silu", "relu"])
@pytest.mark.parametrize("shape", [(64, 2048), (3, 7), (1, 5, 4)])
def test_bias_act_matches_chain(tcx, oracle, act, shape):
    """The fused chain equals the reference's add-then-activation calls."""
    rng = np.random.default_rng(1)
    x = rng.normal(size=shape).astype(np.float32) * 4
    bias = rng.normal(size=shape[-1]).astype(np.float32)
    expected = oracle.add(x, bias)
    if act == "silu":
        expected = oracle.silu(expected)
    elif act == "relu":
        expected = oracle.relu(expected)
    close(host(tcx.bias_act(dev(x), dev(bias), act)), expected, 1e-6)
