"""Device timing helpers: CUDA events on the launching stream, maxima over ranks."""
from __future__ import annotations

from contextlib import contextmanager

import torch
import torch.distributed as dist


def max_over_ranks(value: float, device=None) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device if device is not None else "cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class EventTimer:
    """Accumulates the device time of regions bracketed by start()/stop() (ms)."""

    def __init__(self):
        self.pairs = []

    def start(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs.append([e, None])

    def stop(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs[-1][1] = e

    def total_ms(self) -> float:
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in self.pairs if b is not None)

    def mean_ms(self) -> float:
        n = sum(1 for _, b in self.pairs if b is not None)
        return self.total_ms() / max(n, 1)


@contextmanager
def cuda_region(timer: EventTimer):
    timer.start()
    try:
        yield
    finally:
        timer.stop()
