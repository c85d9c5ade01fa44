"""Test doubles that run this package's optimizers and collective helpers with no process group.

The reference tests its optimizers without processes through mock DTensors, FSDP modules and
device meshes (tests/mocks/fsdp_mock.py, tests/mocks/hdsp_mock.py).  This package's public API
has single-process fallbacks instead, so the doubles here only need to make the environment
look like a machine without ``torch.distributed`` (or with it, but never initialised), and to
stand in for a 2-D device mesh.  Nothing here starts a process or touches a GPU.
"""
from __future__ import annotations

from contextlib import contextmanager
from typing import Dict, Optional, Sequence, Tuple
from unittest import mock


@contextmanager
def no_distributed(available: bool = False):
    """``torch.distributed`` reports itself unavailable (``available=False``) or available but
    not initialised; any collective called anyway raises, so a test fails if a code path that
    should fall back to single-process behaviour talks to a process group."""
    import torch.distributed as dist

    def forbidden(*a, **k):
        raise AssertionError("a collective was called without a process group")

    names = ["all_gather_into_tensor", "all_gather", "all_reduce", "broadcast", "scatter", "barrier",
             "reduce_scatter_tensor", "all_to_all_single"]
    patches = [mock.patch.object(dist, "is_available", lambda: available),
               mock.patch.object(dist, "is_initialized", lambda: False)]
    patches += [mock.patch.object(dist, n, forbidden) for n in names if hasattr(dist, n)]
    for p in patches:
        p.start()
    try:
        yield
    finally:
        for p in reversed(patches):
            p.stop()


class MeshDouble:
    """A 2-D (replicate, shard) device mesh stand-in: shape, dim names and per-dim groups."""

    def __init__(self, shape: Tuple[int, int] = (2, 2), names: Sequence[str] = ("dp_replicate", "fsdp_shard"),
                 device_type: str = "cpu"):
        self.shape = tuple(shape)
        self.mesh_dim_names = tuple(names)
        self.device_type = device_type
        self.ndim = len(self.shape)
        self._groups: Dict[str, Optional[object]] = {n: None for n in self.mesh_dim_names}

    def size(self, dim: int = None):
        if dim is None:
            n = 1
            for s in self.shape:
                n *= s
            return n
        return self.shape[dim]

    def get_group(self, dim=0):
        name = self.mesh_dim_names[dim] if isinstance(dim, int) else dim
        return self._groups.get(name)
