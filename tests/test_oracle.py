"""Pins the CPU oracle (oracle/tcx_oracle.c) to the reference.

1. Against the committed golden fixtures (tests/golden/reference_cpu.npz, produced by
   the reference's own CPU backend): bit-exact for every case.
2. Against the reference itself (oracle/_ref/libtcx_ref.so) on fresh seeded inputs:
   bit-exact, including NaN payloads and signed zeros.
3. The reference's known answers: 2x2 matmul = 19 22 43 50 (cpu_backend.cpp:593-620);
   IEEE ties (test_math_ops.py:86-91); first signed zero (test_math_ops.py:226-234).
"""
import ast
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_cpu.npz")


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def run(impl, op, inputs, kw):
    if op == "attention":
        return impl.attention(inputs["q"], inputs["k"], inputs["v"], inputs.get("mask"), **kw)
    if op == "attention_softmax":
        return impl.attention_softmax(inputs["scores"], kw["shape"], inputs.get("mask"), kw["causal"], kw["scale"])
    if op in ("add", "subtract", "multiply", "divide", "matmul"):
        return getattr(impl, op)(inputs["a"], inputs["b"])
    return getattr(impl, op)(inputs["x"], **kw)


def golden_cases():
    data = np.load(GOLDEN)
    for key, name, op, kw in ast.literal_eval(str(data["index"])):
        inputs = {k.split("_in_")[1]: data[k] for k in data.files if k.startswith(key + "_in_")}
        kw = dict(kw)
        for k in data.files:
            if k.startswith(key + "_kw_"):
                kw[k.split("_kw_")[1]] = data[k]
        yield name, op, inputs, kw, data[key + "_out"]


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_oracle_matches_golden(oracle, case):
    name, op, inputs, kw, expected = case
    actual = run(oracle, op, inputs, kw)
    assert actual.shape == expected.shape
    np.testing.assert_array_equal(bits(actual), bits(expected))


def _random_cases(seed):
    rng = np.random.default_rng(seed)
    for shape in [(5, 33), (2, 3, 65), (130,), (3, 4, 5, 6)]:
        x = rng.normal(size=shape).astype(np.float32) * 3
        x.flat[rng.integers(0, x.size)] = np.float32(x.max())  # ties
        for ax in [None, 0, -1] + ([(0, len(shape) - 1)] if len(shape) > 1 else []):
            for op in ("sum", "max", "mean", "min"):
                yield op, dict(x=x), dict(axis=ax)
        for ax in [0, -1]:
            yield "argmax", dict(x=x), dict(axis=ax)
            for op in ("softmax", "rmsnorm", "layernorm"):
                yield op, dict(x=x), dict(axis=ax)
        for op in ("exp", "gelu", "silu", "relu"):
            yield op, dict(x=x), {}
    xi = rng.integers(-2**31, 2**31 - 1, size=(6, 50), dtype=np.int64).astype(np.int32)
    for ax in [None, 0, 1]:
        for op in ("sum", "max", "min", "argmax"):
            yield op, dict(x=xi), dict(axis=ax)
    yield "matmul", dict(a=rng.uniform(-1, 1, (3, 17, 9)).astype(np.float32),
                         b=rng.uniform(-1, 1, (9, 5)).astype(np.float32)), {}
    yield "add", dict(a=rng.normal(size=(7, 6)).astype(np.float32), b=rng.normal(size=(6,)).astype(np.float32)), {}
    q, k, v = (rng.normal(size=s).astype(np.float32) for s in ((2, 5, 8), (1, 7, 8), (2, 7, 3)))
    yield "attention", dict(q=q, k=k, v=v, mask=rng.random((5, 7)) > 0.3), dict(causal=bool(seed % 2))


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_oracle_matches_reference(oracle, reference, seed):
    for op, inputs, kw in _random_cases(seed):
        expected = run(reference, op, inputs, kw)
        actual = run(oracle, op, inputs, kw)
        assert actual.shape == expected.shape, (op, kw)
        np.testing.assert_array_equal(bits(actual), bits(expected), err_msg=f"{op} {kw}")


def test_oracle_errors_match_reference(oracle, reference):
    x = np.ones((2, 3), np.float32)
    for impl in (oracle, reference):
        with pytest.raises(ValueError):
            impl.sum(x, axis=2)
        with pytest.raises(ValueError):
            impl.max(np.ones((2, 0), np.float32), axis=1)
        with pytest.raises(ValueError):
            impl.rmsnorm(x, axis=-1, eps=-1.0)
        with pytest.raises(ValueError):
            impl.matmul(x, x)
        with pytest.raises(ValueError):
            impl.mean(np.ones((2, 3), np.int32), axis=None)


def test_known_answers(oracle):
    c = oracle.matmul(np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32))
    np.testing.assert_array_equal(c, [[19, 22], [43, 50]])
    a = np.array([[0., -0., 1e-40, -1e-40, np.inf], [np.nan, 2., np.nan, -np.inf, 2.]], np.float32)
    np.testing.assert_array_equal(oracle.argmax(a, 1), np.argmax(a, axis=1).astype(np.int32))
    z = np.array([[0, 0x80000000], [0x80000000, 0]], np.uint32)
    np.testing.assert_array_equal(oracle.min(z.view(np.float32), 1).view(np.uint32), z[:, 0])
    np.testing.assert_array_equal(oracle.argmax(z.view(np.float32), 1), [0, 0])


def test_sequential_sum_error_is_documented(oracle):
    """The CPU sum is sequential float32: its error grows with n, so the full-tensor
    tolerance is stated against both the CPU result and the exact sum."""
    x = np.random.default_rng(0).normal(size=1 << 20).astype(np.float32)
    seq = float(oracle.sum(x))
    exact = oracle.sum_f64(x)
    assert abs(seq - exact) <= 1e-4 * np.abs(x).sum()
