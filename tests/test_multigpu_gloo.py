"""The N > 1 protocol of the full-tensor reductions, on CPU with gloo (world size 2).

Each rank reduces its shard to a 16-byte record (key, bits, global index) exactly as
tcx_sm100_reduce_partial lays it out, the records are all-gathered, and every rank
folds them in rank order as tcx_sm100_reduce_combine does. The per-shard reduction
here is a host emulation (no GPU); the test checks the sharding, global index bases,
cross-shard tie-breaking and rank-order folding against the CPU oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tensorcx_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        x = rng.standard_normal(100_003, dtype=np.float32)
        x[[7, 50_001, 99_999]] = 9.0          # ties in both shards: lowest index wins
        x[12_345] = np.float32(np.nan)        # first NaN wins for max/argmax/min
        xi = rng.integers(-1000, 1000, 100_003).astype(np.int32)
        out = {}
        for name, data, op in [("sum", x, "sum"), ("max", x, "max"), ("min", x, "min"),
                               ("argmax", x, "argmax"), ("isum", xi, "sum"), ("imax", xi, "max")]:
            b, e = shard.shard_range(data.size, rank, world)
            rec = shard.host_partial(data[b:e], op, index_base=b)
            gathered = [torch.zeros(16, dtype=torch.uint8) for _ in range(world)]
            dist.all_gather(gathered, torch.from_numpy(rec.copy()))
            recs = np.stack([g.numpy() for g in gathered])
            out[name] = shard.host_combine(recs, op, data.dtype, data.size)
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_protocol(oracle):
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    rng = np.random.default_rng(0)
    x = rng.standard_normal(100_003, dtype=np.float32)
    x[[7, 50_001, 99_999]] = 9.0
    x[12_345] = np.float32(np.nan)
    xi = rng.integers(-1000, 1000, 100_003).astype(np.int32)
    for r in range(world):
        got = results[r]
        np.testing.assert_array_equal(np.float32(got["max"]).view(np.uint32), oracle.max(x).view(np.uint32))
        np.testing.assert_array_equal(np.float32(got["min"]).view(np.uint32), oracle.min(x).view(np.uint32))
        assert int(got["argmax"]) == int(oracle.argmax(x))
        assert int(got["isum"]) == int(oracle.sum(xi))
        assert int(got["imax"]) == int(oracle.max(xi))
        assert np.isnan(got["sum"]) == np.isnan(oracle.sum(x))


def test_shard_ranges_cover_and_align():
    for n in (0, 1, 5, 4096, 100_003, 1 << 28):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1 and b0 <= e0
            for b, _ in spans:
                assert b % 4 == 0 or b == n  # 16-byte aligned shard starts for float32/int32
