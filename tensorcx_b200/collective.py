"""Cross-GPU full reductions with the exchange inside the kernel.

One process per GPU. Every rank allocates a mailbox on its GPU
(tcx_sm100_mailbox_create), the 64-byte CUDA IPC handles are all-gathered once over
torch.distributed (gloo or NCCL: plumbing only), and each rank maps every peer's
mailbox (tcx_sm100_mailbox_open). A reduction then runs as one stream-ordered call per
rank, tcx_sm100_reduce_sharded: the rank's shard is folded to one 16-byte record, the
record is stored into every mailbox over NVLink peer memory, and the rank's kernel
waits (bounded) for all records of the call's epoch and folds them in rank order, the
same rule as reduce_combine. No collective library call is on the data path.

This replaces, for the multi-GPU path, reduce_partial + all_gather + reduce_combine
(tensorcx_b200.shard describes the record protocol).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._abi import FLOAT32, INT32, OP, check, lib

_HANDLE_BYTES = 64


class PeerReduction:
    """Sharded full reductions over one process group (all ranks on one node).

    Every rank must call `reduce` the same number of times in the same order (the
    call's epoch pairs the records). `wait_limit_s` bounds the in-kernel wait for the
    peers' records; when it expires the device error word is set
    (tcx_sm100_device_error) and the value is undefined.
    """

    def __init__(self, group=None, device: int | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device() if device is None else device
        self.epoch = 0
        self._peers: list[int] = []
        L = lib()
        with torch.cuda.device(self.device):
            box = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * _HANDLE_BYTES)()
            check(L.tcx_sm100_mailbox_create(self.world, ctypes.byref(box), handle))
            self._own = box.value
            local = torch.tensor(bytearray(handle), dtype=torch.uint8)
            if dist.get_backend(group) == "nccl":
                local = local.cuda()
            gathered = [torch.empty_like(local) for _ in range(self.world)]
            dist.all_gather(gathered, local, group=group)
            ptrs = []
            for r, h in enumerate(gathered):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                raw = (ctypes.c_uint8 * _HANDLE_BYTES)(*h.cpu().tolist())
                peer = ctypes.c_void_p()
                check(L.tcx_sm100_mailbox_open(raw, ctypes.byref(peer)))
                self._peers.append(peer.value)
                ptrs.append(peer.value)
        self._mailboxes = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group)  # every mailbox is zeroed and mapped before the first store

    def reduce(self, shard: torch.Tensor, op: str, index_base: int, total_count: int,
               wait_limit_s: float = 2.0) -> torch.Tensor:
        """The reduction of the whole tensor (sum, mean, max, min, argmax) from this
        rank's contiguous shard starting at global index `index_base`; a 0-d tensor
        on this rank's GPU, equal on every rank."""
        if not shard.is_cuda or not shard.is_contiguous():
            raise ValueError("shard must be a contiguous CUDA tensor")
        if shard.dtype not in (torch.float32, torch.int32):
            raise ValueError("CUDA operations only support float32 and int32 on this path")
        dt = FLOAT32 if shard.dtype == torch.float32 else INT32
        out = torch.empty((), dtype=torch.int32 if op == "argmax" else shard.dtype, device=shard.device)
        L = lib()
        ws_bytes = L.tcx_sm100_reduce_workspace_bytes(shard.numel())
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=shard.device)
        self.epoch += 1
        stream = ctypes.c_void_p(torch.cuda.current_stream(shard.device).cuda_stream)
        check(L.tcx_sm100_reduce_sharded(stream, OP[op], dt, ctypes.c_void_p(shard.data_ptr()), shard.numel(),
                                         index_base, self._mailboxes, self.rank, self.world, self.epoch,
                                         int(wait_limit_s * 1e9), total_count, ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(ws.data_ptr()), ws_bytes))
        return out

    def close(self) -> None:
        """Unmaps the peers' mailboxes and frees this rank's (collective: every rank)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)  # no peer still stores into this rank's mailbox
        L = lib()
        with torch.cuda.device(self.device):
            for p in self._peers:
                check(L.tcx_sm100_mailbox_close(ctypes.c_void_p(p)))
            self._peers = []
            if self._own:
                check(L.tcx_sm100_mailbox_free(ctypes.c_void_p(self._own)))
                self._own = None
