"""Host-side sharding of a full-tensor reduction across ranks.

Each rank owns a contiguous span of the flat input (starts aligned to 4 elements, so
shard pointers stay 16-byte aligned for the 128-bit loads), reduces it on its GPU to
one 16-byte `tcx_partial` record with `tcx_sm100_reduce_partial` (global index base =
span start), and the records, gathered in rank order, are folded by
`tcx_sm100_reduce_combine`. The record layout and fold rules are the ones the kernels
use (reduce.cu); `host_partial` / `host_combine` restate them on the host so the
protocol can be exercised without a GPU (multi-process gloo tests).
"""
from __future__ import annotations

import numpy as np

RECORD = np.dtype([("key", "<u4"), ("bits", "<u4"), ("index", "<i8")])


def shard_range(count: int, rank: int, world: int) -> tuple[int, int]:
    per = -(-count // world) if world else count
    per = (per + 3) // 4 * 4
    begin = min(count, rank * per)
    end = min(count, begin + per) if rank < world - 1 else count
    return begin, end


def _key(word: np.ndarray, fp: bool, largest: bool) -> np.ndarray:
    w = word.astype(np.uint32)
    if not fp:
        k = w ^ np.uint32(0x80000000)
        return k if largest else ~k
    nan = (w & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    w = np.where((w & np.uint32(0x7FFFFFFF)) == 0, np.uint32(0), w)
    ordered = np.where(w & np.uint32(0x80000000), ~w, w | np.uint32(0x80000000)).astype(np.uint32)
    k = ordered if largest else ~ordered
    return np.where(nan, np.uint32(0xFFFFFFFF), k).astype(np.uint32)


def host_partial(x: np.ndarray, op: str, index_base: int) -> np.ndarray:
    """The 16-byte record of one shard, as bytes (uint8[16])."""
    fp = x.dtype == np.float32
    rec = np.zeros(1, RECORD)
    words = x.view(np.uint32)
    if op in ("sum", "mean"):
        if fp:
            rec["bits"] = np.float32(x.sum(dtype=np.float64)).view(np.uint32)
        else:
            rec["bits"] = np.uint32(int(words.astype(np.uint64).sum()) & 0xFFFFFFFF)
        rec["index"] = np.iinfo(np.int64).max
    else:
        keys = _key(words, fp, op in ("max", "argmax"))
        best = int(np.argmax(keys))  # first occurrence of the largest key
        rec["key"], rec["bits"], rec["index"] = keys[best], words[best], index_base + best
    return rec.view(np.uint8)


def host_combine(records: np.ndarray, op: str, dtype, total: int):
    """Folds gathered records in rank order; returns the reduction's value."""
    recs = np.ascontiguousarray(records).view(RECORD).reshape(-1)
    fp = np.dtype(dtype) == np.float32
    if op in ("sum", "mean"):
        if fp:
            acc = np.float32(0)
            for r in recs:
                acc = np.float32(acc + np.uint32(r["bits"]).view(np.float32))
            return np.float32(acc / np.float32(total)) if op == "mean" else acc
        acc = 0
        for r in recs:
            acc = (acc + int(r["bits"])) & 0xFFFFFFFF
        return np.uint32(acc).view(np.int32)
    best = None
    for r in recs:
        if best is None or r["key"] > best["key"] or (r["key"] == best["key"] and r["index"] < best["index"]):
            best = r
    if op == "argmax":
        return int(best["index"])
    return np.uint32(best["bits"]).view(np.float32 if fp else np.int32)
