"""Runs one hot-path workload a few times on cuda:0, for profilers (ncu) and quick
timing. Prints the mean device time per call (CUDA events).

    python -m tensorcx_b200.profile matmul --size 4096 [--path tensor|ffma] [--repeat 3]
    python -m tensorcx_b200.profile bmm --batch 64 --size 2048
    python -m tensorcx_b200.profile softmax|rmsnorm|layernorm --rows 16384 --cols 4096
    python -m tensorcx_b200.profile sum|max|min|argmax|mean --n 268435456 [--int32]
    python -m tensorcx_b200.profile attention --batch 32 --rows 2048 --cols 2048 --size 128 [--causal]
    python -m tensorcx_b200.profile sum_axis0 --rows 65536 --cols 4096
    python -m tensorcx_b200.profile sum_axes02 --batch 64 --rows 4096 --cols 1024
"""
from __future__ import annotations

import argparse

import torch

from . import ops


def main():
    p = argparse.ArgumentParser()
    p.add_argument("workload")
    p.add_argument("--size", type=int, default=4096)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--rows", type=int, default=16384)
    p.add_argument("--cols", type=int, default=4096)
    p.add_argument("--n", type=int, default=1 << 28)
    p.add_argument("--int32", action="store_true")
    p.add_argument("--path", default="auto")
    p.add_argument("--repeat", type=int, default=3)
    p.add_argument("--causal", action="store_true")
    a = p.parse_args()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    w = a.workload
    if w == "matmul":
        x = torch.rand(a.size, a.size, device="cuda", generator=g) * 2 - 1
        y = torch.rand(a.size, a.size, device="cuda", generator=g) * 2 - 1
        fn = lambda: ops.matmul(x, y, path=a.path)  # noqa: E731
    elif w == "bmm":
        x = torch.rand(a.batch, a.size, a.size, device="cuda", generator=g) * 2 - 1
        y = torch.rand(a.batch, a.size, a.size, device="cuda", generator=g) * 2 - 1
        bias = torch.randn(a.size, device="cuda", generator=g)
        fn = lambda: ops.matmul(x, y, bias=bias, act="silu", path=a.path)  # noqa: E731
    elif w in ("softmax", "rmsnorm", "layernorm"):
        x = torch.randn(a.rows, a.cols, device="cuda", generator=g) * 3
        f = getattr(ops, w)
        fn = lambda: f(x, axis=-1)  # noqa: E731
    elif w in ("sum", "max", "min", "argmax", "mean"):
        if a.int32:
            x = torch.randint(-1000, 1001, (a.n,), device="cuda", generator=g, dtype=torch.int32)
        else:
            x = torch.randn(a.n, device="cuda", generator=g)
        f = getattr(ops, w)
        fn = lambda: f(x)  # noqa: E731
    elif w == "sum_axis0":
        x = torch.randn(a.rows, a.cols, device="cuda", generator=g)
        fn = lambda: ops.sum(x, axis=0)  # noqa: E731
    elif w == "sum_axes02":
        x = torch.randn(a.batch, a.rows, a.cols, device="cuda", generator=g)
        fn = lambda: ops.sum(x, axis=(0, 2))  # noqa: E731
    elif w == "attention":  # batch = heads, rows = queries, cols = keys, size = features
        q = torch.randn(a.batch, a.rows, a.size, device="cuda", generator=g)
        k = torch.randn(a.batch, a.cols, a.size, device="cuda", generator=g)
        v = torch.randn(a.batch, a.cols, a.size, device="cuda", generator=g)
        fn = lambda: ops.attention(q, k, v, is_causal=a.causal)  # noqa: E731
    else:
        raise SystemExit(f"unknown workload {w}")
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.repeat):
        fn()
    e.record()
    torch.cuda.synchronize()
    print(f"{w}: {s.elapsed_time(e) / a.repeat:.4f} ms per call")


if __name__ == "__main__":
    main()
