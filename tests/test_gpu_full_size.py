"""GPU parity at the full sizes of the benchmark configurations, device-resident as
bench.py runs them, checked through properties that need no full CPU re-run:

* full reductions over 2^28 elements (float32 N(0,1), int32 U[-1000, 1000]): extrema
  planted as exact ties on both sides of the 2-, 4- and 8-way shard boundaries, so
  the answer is known by construction (lowest index wins, cpu_math.cpp:14-21) and the
  oracle confirms it; int32 sums exact modulo 2^32 (uint32 wraparound,
  cpu_backend.cpp:1099-1249), also with an offset that makes the sum wrap; float32
  sums against the CPU's sequential sum and the float64 sum; the same values again
  from per-shard records folded in rank order (the multi-GPU path on one GPU);
* fp32 matmul 8192^3: row blocks at the start, across a 256-row tile boundary and at
  the end against the oracle (cpu::matmul, cpu_backend.cpp:1251-1276), and every
  output element through the checksums C·1 = A·(B·1) and 1ᵀ·C = (1ᵀ·A)·B in float64;
* bmm [64, 2048, 2048]^2 + bias + SiLU: batches 0 and 63 whole against float64, rows
  of them against the oracle's matmul -> add -> silu, and one row of every batch;
* softmax / rmsnorm / layernorm (+ affine) on [16384, 4096] and softmax on
  [4096, 32768]: sampled rows against the oracle (reference tolerance 1e-5, or closer
  to float64 than the CPU), and row invariants over every row (softmax rows sum to 1,
  normalized rows have the mean and mean square the formulas give).
"""
import math

import numpy as np
import pytest
import torch

from tensorcx_b200 import shard as sharding

pytestmark = pytest.mark.gpu

N28 = 1 << 28


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    if a.dtype == np.float32:
        assert a.view(np.uint32) == b.astype(np.float32).view(np.uint32), (a, b)
    else:
        assert int(a) == int(b), (a, b)


def sum_close(got, cpu, exact):
    """Within 1e-5 relative of the CPU's sequential float32 sum, or closer to the exact
    sum than that CPU result is (the sequential sum is not the more accurate one)."""
    return abs(got - cpu) <= 1e-5 * abs(cpu) or abs(got - exact) <= abs(cpu - exact)


def frob_rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.linalg.norm((got - ref).ravel()) / max(np.linalg.norm(ref.ravel()), 1e-300)


def matmul_tol(k):
    return 1e-4 * math.sqrt(max(k, 1024) / 1024)


def boundary_ties(n):
    """Positions straddling shard boundaries for 2, 4 and 8 shards, lowest first."""
    edges = sorted({sharding.shard_range(n, r, w)[0] for w in (2, 4, 8) for r in range(1, w)})
    mx = [edges[2] - 1, edges[2], edges[5], n - 1]  # lowest index: one before an 8-way edge
    mn = [edges[0] - 1, edges[0], edges[3] + 1]
    return mx, mn


def sharded(tcx, xd, op, world):
    """The multi-GPU reduction emulated on one GPU: each shard's record, folded in
    rank order by the combine kernel."""
    n = xd.numel()
    recs = []
    for r in range(world):
        b, e = sharding.shard_range(n, r, world)
        recs.append(tcx.reduce_partial(xd[b:e], op, index_base=b))
    return tcx.reduce_combine(torch.stack(recs), op, xd.dtype, n)


def test_full_reductions_float32_2e28(tcx, oracle):
    x = np.random.default_rng(0).standard_normal(N28, dtype=np.float32)
    mx, mn = boundary_ties(N28)
    top, bottom = np.float32(x.max() + 1), np.float32(x.min() - 1)
    x[mx] = top
    x[mn] = bottom
    xd = dev(x)
    assert int(host(tcx.argmax(xd))) == mx[0] == int(oracle.argmax(x))
    same_bits(host(tcx.max(xd)), top)
    same_bits(host(tcx.min(xd)), bottom)
    cpu_sum, exact = float(oracle.sum(x)), oracle.sum_f64(x)
    got_sum = float(host(tcx.sum(xd)))
    assert sum_close(got_sum, cpu_sum, exact), (got_sum, cpu_sum, exact)
    got_mean = float(host(tcx.mean(xd)))
    assert sum_close(got_mean, float(oracle.mean(x)), exact / N28), (got_mean, exact / N28)
    for world in (2, 8):
        assert int(host(sharded(tcx, xd, "argmax", world))) == mx[0]
        same_bits(host(sharded(tcx, xd, "max", world)), top)
        same_bits(host(sharded(tcx, xd, "min", world)), bottom)
        s = float(host(sharded(tcx, xd, "sum", world)))
        assert sum_close(s, cpu_sum, exact), (world, s, cpu_sum, exact)


def test_full_reductions_int32_2e28(tcx, oracle):
    x = np.random.default_rng(1).integers(-1000, 1001, N28, dtype=np.int32)
    mx, mn = boundary_ties(N28)
    x[mx] = 1001
    x[mn] = -1001
    xd = dev(x)

    def wrapped(v):
        return np.int64(np.sum(v, dtype=np.int64)).astype(np.uint64).astype(np.uint32).view(np.int32)

    assert int(host(tcx.sum(xd))) == int(wrapped(x))
    assert int(host(tcx.max(xd))) == 1001
    assert int(host(tcx.min(xd))) == -1001
    assert int(host(tcx.argmax(xd))) == mx[0]
    for world in (2, 8):
        assert int(host(sharded(tcx, xd, "sum", world))) == int(wrapped(x))
        assert int(host(sharded(tcx, xd, "argmax", world))) == mx[0]
    # an offset of 2^23 per element makes the 2^28-element sum wrap around 2^32 many times
    xd += 1 << 23
    x += 1 << 23
    want = wrapped(x)
    assert int(host(tcx.sum(xd))) == int(want)
    assert int(host(sharded(tcx, xd, "sum", 8))) == int(want)
    assert int(oracle.sum(x[:1 << 20])) == int(wrapped(x[:1 << 20]))  # the oracle wraps the same way


def test_matmul_8192_cube(tcx, oracle):
    n = 8192
    rng = np.random.default_rng(8192)
    a = rng.random((n, n), dtype=np.float32) * 2 - 1
    b = rng.random((n, n), dtype=np.float32) * 2 - 1
    cd = tcx.matmul(dev(a), dev(b))
    tol = matmul_tol(n)
    b64 = b.astype(np.float64)
    for rows in (slice(0, 4), slice(4094, 4098), slice(n - 4, n)):
        got = host(cd[rows])
        ref = oracle.matmul(a, b, rows=rows, batches=[0])[0]
        assert frob_rel(got, ref) <= tol, (rows, frob_rel(got, ref))
        exact = a[rows].astype(np.float64) @ b64
        assert frob_rel(got, exact) <= tol, (rows, frob_rel(got, exact))
    # every output element: row and column checksums in float64
    row_sums = host(cd.double().sum(dim=1))
    want_rows = a.astype(np.float64) @ np.sum(b, axis=1, dtype=np.float64)
    assert frob_rel(row_sums, want_rows) <= tol, frob_rel(row_sums, want_rows)
    col_sums = host(cd.double().sum(dim=0))
    want_cols = np.sum(a, axis=0, dtype=np.float64) @ b64
    assert frob_rel(col_sums, want_cols) <= tol, frob_rel(col_sums, want_cols)
    assert torch.isfinite(cd).all()


def silu64(z):
    return z / (1.0 + np.exp(-z))


def test_bmm_64x2048_bias_silu(tcx, oracle):
    nb, n = 64, 2048
    rng = np.random.default_rng(64)
    a = rng.random((nb, n, n), dtype=np.float32) * 2 - 1
    b = rng.random((nb, n, n), dtype=np.float32) * 2 - 1
    bias = rng.standard_normal(n, dtype=np.float32)
    cd = tcx.matmul(dev(a), dev(b), bias=dev(bias), act="silu")
    tol = matmul_tol(n)
    for i in (0, nb - 1):
        got = host(cd[i])
        exact = silu64(a[i].astype(np.float64) @ b[i].astype(np.float64) + bias)
        assert frob_rel(got, exact) <= tol, (i, frob_rel(got, exact))
        rows = slice(1020, 1030)
        ref = oracle.silu(oracle.add(oracle.matmul(a, b, rows=rows, batches=[i])[0], bias))
        assert frob_rel(got[rows], ref) <= tol, (i, frob_rel(got[rows], ref))
    picks = [(37 * i) % n for i in range(nb)]  # one row of every batch
    got = host(cd[torch.arange(nb, device="cuda"), torch.tensor(picks, device="cuda")])
    exact = np.stack([silu64(a[i, r].astype(np.float64) @ b[i].astype(np.float64) + bias)
                      for i, r in enumerate(picks)])
    assert frob_rel(got, exact) <= tol, frob_rel(got, exact)


def exact_rows(op, x, eps=1e-5):
    x = x.astype(np.float64)
    if op == "softmax":
        e = np.exp(x - x.max(axis=-1, keepdims=True))
        return e / e.sum(axis=-1, keepdims=True)
    if op == "rmsnorm":
        return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + np.float32(eps))
    m = x.mean(axis=-1, keepdims=True)
    return (x - m) / np.sqrt(np.mean((x - m) ** 2, axis=-1, keepdims=True) + np.float32(eps))


def rows_close(got, cpu, exact, tol=1e-5):
    got, cpu, exact = (np.asarray(v, np.float64) for v in (got, cpu, exact))
    near = np.abs(got - cpu) <= tol + tol * np.abs(cpu)
    better = np.abs(got - exact) <= np.abs(cpu - exact) + 1e-7 * np.abs(exact)
    bad = ~(near | better)
    assert not bad.any(), (got[bad][:5], cpu[bad][:5], exact[bad][:5])


def sample_rows(r):
    return np.r_[0:4, r // 2 - 2:r // 2 + 2, r - 4:r]


@pytest.mark.parametrize("rows,cols", [(16384, 4096), (4096, 32768)])
def test_row_ops_full(tcx, oracle, rows, cols):
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, cols), dtype=np.float32) * 3
    xd = dev(x)
    pick = sample_rows(rows)
    ops = ["softmax"] if cols > 4096 else ["softmax", "rmsnorm", "layernorm"]
    eps = 1e-5
    x64 = xd.double()
    for op in ops:
        yd = tcx.softmax(xd, axis=-1) if op == "softmax" else getattr(tcx, op)(xd, axis=-1, eps=eps)
        xs = x[pick]
        cpu = oracle.softmax(xs, -1) if op == "softmax" else getattr(oracle, op)(xs, -1, eps)
        rows_close(host(yd[torch.from_numpy(pick).cuda()]), cpu, exact_rows(op, xs, eps))
        y = yd.double()
        if op == "softmax":
            assert (yd >= 0).all() and (yd <= 1).all()
            assert (y.sum(dim=1) - 1).abs().max().item() <= 1e-5
        elif op == "rmsnorm":
            ms = (x64 * x64).mean(dim=1)
            want = ms / (ms + np.float32(eps))
            assert ((y * y).mean(dim=1) - want).abs().max().item() <= 1e-5
        else:
            assert y.mean(dim=1).abs().max().item() <= 1e-5
            var = x64.var(dim=1, unbiased=False)
            want = var / (var + np.float32(eps))
            assert (y.var(dim=1, unbiased=False) - want).abs().max().item() <= 1e-5
        del yd, y
    if cols == 4096:  # the affine forms of config 3: gamma ~ U(0.5, 1.5), beta ~ N(0, 0.1)
        g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        beta = (rng.standard_normal(cols) * 0.1).astype(np.float32)
        yd = tcx.layernorm(xd, axis=-1, eps=eps, weight=dev(g), bias=dev(beta))
        xs = x[pick]
        cpu = oracle.layernorm(xs, -1, eps, g, beta)
        exact = exact_rows("layernorm", xs, eps) * g.astype(np.float64) + beta.astype(np.float64)
        rows_close(host(yd[torch.from_numpy(pick).cuda()]), cpu, exact)
        z = (yd.double() - dev(beta).double()) / dev(g).double()
        assert z.mean(dim=1).abs().max().item() <= 1e-5
        yd = tcx.rmsnorm(xd, axis=-1, eps=eps, weight=dev(g))
        rows_close(host(yd[torch.from_numpy(pick).cuda()]), oracle.rmsnorm(xs, -1, eps, g),
                   exact_rows("rmsnorm", xs, eps) * g.astype(np.float64))
