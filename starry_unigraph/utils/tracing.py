"""Tracing and timing helpers (the reference only used time.perf_counter and
per-step millisecond fields, backends/ctdg/runtime/runtime.py:241-327).

* ``nvtx_range(name)``: NVTX range around a phase (sample / fetch / attention /
  update / push / backward / all-reduce), visible in Nsight timelines; a no-op
  without CUDA.
* ``DeviceTimer``: CUDA-event timing on the current stream.
* ``max_over_ranks(x)``: the slowest rank's value (the metric the framework
  reports for multi-GPU timings).
"""
from __future__ import annotations

import contextlib
import time
from typing import Iterator

import torch
import torch.distributed as dist


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    use = torch.cuda.is_available()
    if use:
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if use:
            torch.cuda.nvtx.range_pop()


class DeviceTimer:
    """Milliseconds between start() and stop() on the device (CUDA events), or
    wall-clock milliseconds on CPU."""

    def __init__(self) -> None:
        self.cuda = torch.cuda.is_available()
        self._t0 = 0.0
        if self.cuda:
            self._a = torch.cuda.Event(enable_timing=True)
            self._b = torch.cuda.Event(enable_timing=True)

    def start(self) -> "DeviceTimer":
        if self.cuda:
            self._a.record()
        else:
            self._t0 = time.perf_counter()
        return self

    def stop(self) -> float:
        if self.cuda:
            self._b.record()
            self._b.synchronize()
            return float(self._a.elapsed_time(self._b))
        return (time.perf_counter() - self._t0) * 1000.0


def max_over_ranks(value: float) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
