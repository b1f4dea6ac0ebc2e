"""Generates tests/golden/*.npz from the reference's own CPU backend.

    python tests/golden/make_golden.py

Inputs are seeded (numpy default_rng); outputs come from oracle/_ref/libtcx_ref.so,
which oracle/Makefile compiles from the tensor.cx sources (cpp/tensorcx/core and
backends/cpu). The fixtures pin the C restatement (oracle/tcx_oracle.c) to the
reference on machines where the reference tree is absent. Cases mirror the
reference's own tests for this path: tests/python/test_cuda_primitives.py (shapes,
special values, constant rows, staged widths), test_math_ops.py (IEEE ties, signed
zeros), test_batched_matmul.py (broadcast batches, special values) and the 2x2
known answer of cpu_backend.cpp:593-620.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.oracle import Reference  # noqa: E402


def cases():
    rng = np.random.default_rng(20260101)
    f = lambda *s, scale=1.0: (rng.normal(size=s) * scale).astype(np.float32)  # noqa: E731
    special_rows = np.array([[0., -0., 1e-38, -1e-38], [1., np.nan, 2., 3.], [np.inf, 1., 2., -np.inf],
                             [1e20] * 4], np.float32)
    ties = np.array([[0., -0., 1e-40, -1e-40, np.inf], [np.nan, 2., np.nan, -np.inf, 2.]], np.float32)
    zeros = np.array([[0, 0x80000000], [0x80000000, 0]], np.uint32).view(np.float32)
    out = []
    for shape in [(), (1,), (7,), (2, 3, 5), (4, 257), (3, 1100), (2, 3, 255)]:
        x = f(*shape)
        for ax in ([None] + list(range(-len(shape), len(shape)))) if shape else [None, 0]:
            for op in ("sum", "max", "mean"):
                out.append((f"{op}_{shape}_{ax}", op, dict(x=x), dict(axis=ax)))
    for op in ("sum", "max"):
        xi = rng.integers(-1000, 1000, size=(5, 300)).astype(np.int32)
        for ax in (None, 0, 1):
            out.append((f"{op}_i32_{ax}", op, dict(x=xi), dict(axis=ax)))
        big = np.full((3, 7), 2**30, np.int32)
        out.append((f"{op}_i32_wrap", op, dict(x=big), dict(axis=None)))
    for name, x in (("special", special_rows), ("ties", ties), ("zeros", zeros),
                    ("rand", f(4, 9)), ("ints", rng.integers(-3, 4, (2, 3, 4)).astype(np.float32))):
        for ax in (None, 0, 1, -1):
            out.append((f"min_{name}_{ax}", "min", dict(x=x), dict(axis=ax)))
            out.append((f"argmax_{name}_{ax}", "argmax", dict(x=x), dict(axis=ax)))
    xi = rng.integers(-3, 4, (2, 3, 4)).astype(np.int32)
    for ax in (None, 0, 1, -1):
        out.append((f"argmax_i32_{ax}", "argmax", dict(x=xi), dict(axis=ax)))
        out.append((f"min_i32_{ax}", "min", dict(x=xi), dict(axis=ax)))
    for op in ("softmax", "rmsnorm", "layernorm"):
        for shape, ax in [((2, 3, 5), -1), ((2, 3, 5), 0), ((4, 300), -1), ((2, 33), 1), ((7,), 0)]:
            out.append((f"{op}_{shape}_{ax}", op, dict(x=f(*shape, scale=3.0)), dict(axis=ax)))
        out.append((f"{op}_special", op, dict(x=special_rows.T.copy()), dict(axis=0)))
    for op in ("rmsnorm", "layernorm"):
        for eps in (0.0, 1e-45, 1e-5, 1e30):
            for value in (0.0, 0.3, 1e38):
                out.append((f"{op}_const_{eps}_{value}", op, dict(x=np.full((2, 33), value, np.float32)),
                            dict(axis=-1, eps=eps)))
    x = f(3, 8, 64, scale=3.0)
    w = rng.uniform(0.5, 1.5, 64).astype(np.float32)
    b = (rng.normal(size=64) * 0.1).astype(np.float32)
    out.append(("layernorm_affine", "layernorm", dict(x=x), dict(axis=-1, eps=1e-5, weight=w, bias=b)))
    out.append(("rmsnorm_affine", "rmsnorm", dict(x=x), dict(axis=-1, eps=1e-5, weight=w)))
    grid = np.linspace(-8, 8, 257, dtype=np.float32)
    specials = np.array([0., -0., np.inf, -np.inf, np.nan, 100, -100, 1e-38], np.float32)
    for op in ("exp", "gelu", "silu"):
        out.append((f"{op}_grid", op, dict(x=grid), {}))
        out.append((f"{op}_special", op, dict(x=specials), {}))
    out.append(("relu_special", "relu", dict(x=np.concatenate([specials, grid])), {}))
    for op in ("add", "subtract", "multiply", "divide"):
        out.append((f"{op}_bcast", op, dict(a=f(4, 1, 6), b=f(3, 1)), {}))
    out.append(("add_bias", "add", dict(a=f(16, 10), b=f(10)), {}))
    out.append(("add_i32_wrap", "add", dict(a=np.full((4,), 2**31 - 1, np.int32), b=np.ones((4,), np.int32)), {}))
    out.append(("matmul_2x2", "matmul", dict(a=np.array([[1, 2], [3, 4]], np.float32),
                                             b=np.array([[5, 6], [7, 8]], np.float32)), {}))
    for sa, sb in [((3,), (3,)), ((2, 3), (3,)), ((3,), (3, 4)), ((2, 3, 4), (2, 4, 5)), ((2, 3, 4), (4, 5)),
                   ((2, 1, 3, 4), (1, 5, 4, 6)), ((2, 17, 19), (1, 19, 33)), ((15, 17), (17, 31)),
                   ((65, 129), (129, 67))]:
        out.append((f"matmul_{sa}_{sb}", "matmul", dict(a=rng.uniform(-1, 1, sa).astype(np.float32),
                                                        b=rng.uniform(-1, 1, sb).astype(np.float32)), {}))
    a = np.array([[[np.nan, 1]], [[np.inf, 1]], [[-np.inf, -1]], [[-0., 0.]]], np.float32)
    out.append(("matmul_special", "matmul", dict(a=a, b=np.array([[1.], [2.]], np.float32)), {}))
    # attention composite and primitive (test_inference_ops.py:27-164 shapes and masks)
    g = np.random.default_rng(20260102)
    n = lambda *s: g.normal(size=s).astype(np.float32)  # noqa: E731
    for sq, sk, sv in [((3, 4), (5, 4), (5, 2)), ((2, 3, 4), (2, 5, 4), (2, 5, 6)),
                       ((2, 1, 3, 4), (1, 3, 5, 4), (2, 3, 5, 2)), ((3, 4), (5, 4), (2, 1, 5, 2)),
                       ((0, 4), (5, 4), (5, 2)), ((3, 4), (0, 4), (0, 2)), ((3, 4), (5, 4), (5, 0))]:
        lq, lk = sq[-2], sk[-2]
        bool_mask = g.random((lq, lk)) > 0.4
        if lq:
            bool_mask[0] = False
        add_mask = n(lq, lk)
        add_mask[g.random((lq, lk)) < 0.3] = -np.inf
        for mname, mask in (("none", None), ("bool", bool_mask), ("add", add_mask), ("false", np.array(False))):
            for causal in (False, True):
                ins = dict(q=n(*sq), k=n(*sk), v=n(*sv))
                if mask is not None:
                    ins["mask"] = mask
                out.append((f"attention_{sq}_{sk}_{mname}_{causal}", "attention", ins, dict(causal=causal)))
    for scale in (0.0, -0.5, 2.0, 1e-40):
        out.append((f"attention_scale_{scale}", "attention",
                    dict(q=n(2, 3, 4), k=n(5, 4), v=n(5, 3), mask=g.random((2, 1, 5)) > 0.3), dict(scale=scale)))
    k = np.ones((2, 2), np.float32)
    k[0] = np.nan
    out.append(("attention_nan_key", "attention", dict(q=np.ones((1, 2), np.float32), k=k, v=n(2, 3)), {}))
    for shape, sshape, mshape, causal in [((2, 3, 7), (3, 7), (2, 1, 7), True), ((4, 9), (4, 1), (9,), False)]:
        mask = n(*mshape)
        mask[g.random(mshape) < 0.3] = -np.inf
        out.append((f"attention_softmax_{shape}", "attention_softmax", dict(scores=n(*sshape), mask=mask),
                    dict(shape=shape, causal=causal, scale=0.7)))
    return out


def run(ref, op, inputs, kw):
    if op == "attention":
        return ref.attention(inputs["q"], inputs["k"], inputs["v"], inputs.get("mask"), **kw)
    if op == "attention_softmax":
        return ref.attention_softmax(inputs["scores"], kw["shape"], inputs.get("mask"), kw["causal"], kw["scale"])
    if op in ("add", "subtract", "multiply", "divide", "matmul"):
        return getattr(ref, op)(inputs["a"], inputs["b"])
    return getattr(ref, op)(inputs["x"], **kw)


def main():
    ref = Reference()
    arrays = {}
    index = []
    for i, (name, op, inputs, kw) in enumerate(cases()):
        key = f"c{i:03d}"
        for k, v in inputs.items():
            arrays[f"{key}_in_{k}"] = v
        for k, v in kw.items():
            if isinstance(v, np.ndarray):
                arrays[f"{key}_kw_{k}"] = v
        arrays[f"{key}_out"] = run(ref, op, inputs, kw)
        index.append((key, name, op, {k: v for k, v in kw.items() if not isinstance(v, np.ndarray)}))
    arrays["index"] = np.array(repr(index))
    np.savez_compressed(os.path.join(HERE, "reference_cpu.npz"), **arrays)
    print(f"{len(index)} cases -> reference_cpu.npz")


if __name__ == "__main__":
    main()
