"""Replaying a fixed sequence of ops as one CUDA graph.

Every op of this package is stream-ordered on the caller's current stream, never
synchronises the host, and takes its scratch space from torch's caching allocator (the
C ABI itself never allocates), so a sequence of them captures into a CUDA graph as it
stands. A replay then costs one graph launch instead of one host round trip per op
(argument checks, shape planning and the ctypes call of each op), which is what bounds
small, latency-bound sequences such as a 2-layer MLP forward.

The captured graph reads the tensors that the sequence read during capture and writes
the tensors it returned: update inputs in place (`x.copy_(new)`) and read the returned
tensors after each replay; they are overwritten by the next one.
"""
from __future__ import annotations

from typing import Any, Callable

import torch


class CapturedSequence:
    """`fn()` run `warmup` times on a side stream (first-call setup such as kernel
    attributes happens there), then captured once; calling the object replays it on
    the current stream and returns what `fn` returned at capture."""

    def __init__(self, fn: Callable[[], Any], warmup: int = 2):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA graphs need a CUDA device")
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = fn()

    def __call__(self) -> Any:
        self.graph.replay()
        return self.outputs

    def release(self) -> None:
        """Frees the graph and its private memory pool."""
        self.graph.reset()
        self.outputs = None
