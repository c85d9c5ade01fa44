"""NVTX ranges around the library's fused paths (visible in Nsight Systems / ncu range filters).

The reference has no tracing (it only suggests ``torch.profiler`` in docs/performance.md:365-379).
Here every hot path opens a named range: the Muon step phases (momentum, exchange, Newton–Schulz
per shape group, apply), the fused FSDP collectives (all-gather GEMM, reduce-scatter), attention
forward/backward and the trainer's micro-batches and optimizer steps.

Ranges cost a host call each, so they are off unless ``MMF_NVTX=1`` is set (or ``enable()`` is
called); when off, ``nvtx_range`` is a no-op context manager.
"""
from __future__ import annotations

import contextlib
import os
from typing import Iterator

import torch

_ENABLED = os.environ.get("MMF_NVTX", "0") not in ("", "0", "false", "False")


def enable(flag: bool = True) -> None:
    global _ENABLED
    _ENABLED = bool(flag)


def enabled() -> bool:
    return _ENABLED


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not _ENABLED or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
