"""The multi-GPU full reduction with its exchange in the kernel (tcx_sm100_reduce_sharded,
tensorcx_b200.collective.PeerReduction), against the record path it replaces:
reduce_partial on each shard, the records gathered in rank order, reduce_combine.
The results must be bit-identical (same per-shard arithmetic, same rank-order fold).

On one GPU: world size 1 through the mailbox, and the bounded wait running out (a
second mailbox slot that no rank ever fills) with the error reported on the host.
With 2, 4 or 8 GPUs: one process per GPU exchanges over NVLink peer memory, and the
result is checked against the record path and against the CPU oracle over the whole
array.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

OPS = [("sum", np.float32), ("mean", np.float32), ("max", np.float32), ("min", np.float32),
       ("argmax", np.float32), ("sum", np.int32), ("max", np.int32)]


def _data(dtype, n, seed):
    rng = np.random.default_rng(seed)
    if dtype == np.int32:
        return rng.integers(-1000, 1001, n).astype(np.int32)
    x = rng.standard_normal(n, dtype=np.float32)
    x[[11, n // 2 + 3, n - 5]] = 7.5  # equal maxima in both halves: the lowest index wins
    return x


def _record_path(tcx, shards, bases, op, dtype, total):
    recs = torch.stack([tcx.reduce_partial(s, op, index_base=b) for s, b in zip(shards, bases)])
    return tcx.reduce_combine(recs, op, torch.float32 if dtype == np.float32 else torch.int32, total)


def _sharded(lib, x, op, base, mailboxes, rank, world, epoch, total, limit_ns):
    from tensorcx_b200._abi import FLOAT32, INT32, OP, check
    out = torch.empty((), dtype=torch.int32 if op == "argmax" else x.dtype, device=x.device)
    ws_bytes = lib.tcx_sm100_reduce_workspace_bytes(x.numel())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    boxes = (ctypes.c_void_p * world)(*mailboxes)
    check(lib.tcx_sm100_reduce_sharded(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), OP[op],
                                       FLOAT32 if x.dtype == torch.float32 else INT32,
                                       ctypes.c_void_p(x.data_ptr()), x.numel(), base, boxes, rank, world, epoch,
                                       limit_ns, total, ctypes.c_void_p(out.data_ptr()),
                                       ctypes.c_void_p(ws.data_ptr()), ws_bytes))
    return out


def _mailbox(lib, world):
    from tensorcx_b200._abi import check
    box = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * 64)()
    check(lib.tcx_sm100_mailbox_create(world, ctypes.byref(box), handle))
    return box.value


@pytest.mark.parametrize("op,dtype", OPS)
def test_single_rank_exchange_matches_record_path(tcx, op, dtype):
    from tensorcx_b200 import _abi
    lib = _abi.lib()
    x = torch.from_numpy(_data(dtype, 1_000_003, 3)).cuda()
    box = _mailbox(lib, 1)
    try:
        for epoch in (1, 2, 3):  # both slot sets, reused
            got = _sharded(lib, x, op, 0, [box], 0, 1, epoch, x.numel(), 0)
            want = _record_path(tcx, [x], [0], op, dtype, x.numel())
            torch.cuda.synchronize()
            assert got.cpu().numpy().tobytes() == want.cpu().numpy().tobytes(), (op, epoch)
        code = ctypes.c_int(-1)
        assert lib.tcx_sm100_device_error(0, ctypes.byref(code)) == 0 and code.value == 0
    finally:
        torch.cuda.synchronize()
        lib.tcx_sm100_mailbox_free(ctypes.c_void_p(box))


def test_missing_peer_times_out_with_an_error(tcx):
    """World size 2 where rank 1 never publishes: the kernel's wait runs out after
    0.2 s, the device error word says so, and the library keeps working."""
    from tensorcx_b200 import _abi
    lib = _abi.lib()
    x = torch.randn(4096, device="cuda")
    own, absent = _mailbox(lib, 2), _mailbox(lib, 2)
    try:
        code = ctypes.c_int(0)
        lib.tcx_sm100_device_error(0, ctypes.byref(code))  # clear
        _sharded(lib, x, "sum", 0, [own, absent], 0, 2, 1, 2 * x.numel(), 200_000_000)
        torch.cuda.synchronize()
        assert lib.tcx_sm100_device_error(0, ctypes.byref(code)) == 0
        assert code.value == 0x501
        s = float(tcx.sum(x).item())
        assert np.isfinite(s)
        assert lib.tcx_sm100_device_error(0, ctypes.byref(code)) == 0 and code.value == 0
    finally:
        torch.cuda.synchronize()
        lib.tcx_sm100_mailbox_free(ctypes.c_void_p(own))
        lib.tcx_sm100_mailbox_free(ctypes.c_void_p(absent))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from tensorcx_b200 import ops, shard
    from tensorcx_b200.collective import PeerReduction
    out = {}
    peer = PeerReduction()
    try:
        for i, (op, dtype) in enumerate(OPS * 2):
            full = _data(dtype, 3_000_017, 17 + i)
            b, e = shard.shard_range(full.size, rank, world)
            x = torch.from_numpy(full[b:e].copy()).cuda()
            got = peer.reduce(x, op, b, full.size, wait_limit_s=5.0)
            rec = ops.reduce_partial(x, op, index_base=b).cpu()
            gathered = [torch.zeros(16, dtype=torch.uint8) for _ in range(world)]
            dist.all_gather(gathered, rec)
            want = ops.reduce_combine(torch.stack(gathered).cuda(), op,
                                      torch.float32 if dtype == np.float32 else torch.int32, full.size)
            torch.cuda.synchronize()
            out[f"{i}:{op}:{np.dtype(dtype).name}"] = (got.cpu().numpy().tobytes(), want.cpu().numpy().tobytes())
        code = ctypes.c_int(-1)
        from tensorcx_b200 import _abi
        _abi.lib().tcx_sm100_device_error(rank, ctypes.byref(code))
        out["device_error"] = code.value
    finally:
        peer.close()
        dist.destroy_process_group()
    results[rank] = out


def _check_against_oracle(oracle, op, dtype, full, got_bytes):
    """The multi-GPU result against the CPU oracle over the whole array: bit-exact for
    int32, max, min and argmax (lowest index of the planted cross-shard ties); float32
    sum and mean within 1e-5 relative of the CPU's sequential result, or closer to the
    float64 sum than that result."""
    out_dtype = np.int32 if (op == "argmax" or dtype == np.int32) else np.float32
    got = np.frombuffer(got_bytes, dtype=out_dtype)[0]
    want = np.asarray(getattr(oracle, op)(full)).reshape(())
    if op in ("sum", "mean") and dtype == np.float32:
        exact = oracle.sum_f64(full) / (full.size if op == "mean" else 1)
        assert abs(float(got) - float(want)) <= 1e-5 * abs(float(want)) or \
            abs(float(got) - exact) <= abs(float(want) - exact), (op, float(got), float(want), exact)
    else:
        assert got.tobytes() == want.astype(out_dtype).tobytes(), (op, got, want)
    if op == "argmax":
        assert int(got) == 11  # the first of the planted equal maxima, in shard 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_exchange_matches_record_path_and_oracle(oracle, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        res = dict(results[r])
        assert res.pop("device_error") == 0
        for key, (got, want) in res.items():
            assert got == want, (r, key)
    # every rank holds the same values
    for r in range(1, world):
        assert dict(results[0]) == dict(results[r])
    # and they are the reference's values for the whole array
    res = dict(results[0])
    res.pop("device_error")
    for i, (op, dtype) in enumerate(OPS * 2):
        full = _data(dtype, 3_000_017, 17 + i)
        got, _ = res[f"{i}:{op}:{np.dtype(dtype).name}"]
        _check_against_oracle(oracle, op, dtype, full, got)
