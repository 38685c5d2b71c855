"""NVTX ranges for profiler timelines, off unless VMC_NVTX=1.

Ranges: ``engine.step <n>`` around each engine step, ``layer <i>`` around each layer of an eager
forward (a decode step replayed from a CUDA graph has no host code between kernels, so only its
engine-step range appears), and ``allreduce`` around the TP collectives. The reference has no
profiler annotations (its per-forward log lines are src/core/engine.cpp:1267-1274).
"""
from __future__ import annotations

import contextlib
import os

ENABLED = os.environ.get("VMC_NVTX", "") == "1"


class _TorchBackend:
    @staticmethod
    def push(name: str) -> None:
        import torch
        torch.cuda.nvtx.range_push(name)

    @staticmethod
    def pop() -> None:
        import torch
        torch.cuda.nvtx.range_pop()


backend = _TorchBackend()


@contextlib.contextmanager
def nvtx_range(name: str):
    if not ENABLED:
        yield
        return
    backend.push(name)
    try:
        yield
    finally:
        backend.pop()


class LayerRanges:
    """`next(i)` closes the previous layer's range and opens layer i's; `close()` ends the last one.
    Suits loops whose body leaves through several `continue`s."""

    def __init__(self):
        self.open = False

    def next(self, i: int) -> None:
        if not ENABLED:
            return
        if self.open:
            backend.pop()
        backend.push(f"layer {i}")
        self.open = True

    def close(self) -> None:
        if self.open:
            backend.pop()
            self.open = False
