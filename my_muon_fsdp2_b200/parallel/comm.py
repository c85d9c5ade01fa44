"""Collective primitives with single-process fallbacks.

API parity with the reference's two comm layers:
``src/fsdp2_utils/comm.py:18-267`` (is_distributed, get_world_size, get_rank, get_local_rank,
all_gather, all_gather_grads, scatter, scatter_updates, all_reduce, all_reduce_sum,
all_reduce_avg, broadcast, barrier) and ``src/muon_fsdp/distributed.py:13-170``
(is_available, all_gather_grads, scatter_updates).

Differences (deliberate):
* ``scatter_updates`` works (the reference passes an unsupported ``src_tensor=`` kwarg,
  distributed.py:161-166) and, because every rank already holds the identical full update in
  the NS-replication scheme, it slices locally instead of shipping data from rank 0.
* Rows that do not divide by the world size follow ``torch.chunk`` (FSDP2's own sharding)
  instead of raising.
* Gathers are bucketed: all tensors of one dtype go through a single
  ``all_gather_into_tensor`` instead of one collective per tensor.
"""
from __future__ import annotations

import os
from collections import OrderedDict
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def is_available() -> bool:
    """True when torch.distributed is available *and* initialised."""
    return dist.is_available() and dist.is_initialized()


is_distributed = is_available


def get_world_size(group: Optional[dist.ProcessGroup] = None) -> int:
    return dist.get_world_size(group) if is_available() else 1


def get_rank(group: Optional[dist.ProcessGroup] = None) -> int:
    return dist.get_rank(group) if is_available() else 0


def get_local_rank() -> int:
    """Rank within the node (LOCAL_RANK from the launcher, else the global rank)."""
    if not is_available():
        return 0
    lr = os.environ.get("LOCAL_RANK")
    if lr is not None:
        return int(lr)
    try:
        return dist.get_node_local_rank()  # torch >= 2.4
    except Exception:
        return get_rank()


def chunk_rows(rows: int, world: int) -> List[int]:
    """Row counts per rank under ``torch.chunk`` semantics (FSDP2's Shard(0) layout)."""
    cs = (rows + world - 1) // world if world > 0 else rows
    out = []
    for r in range(world):
        lo = min(r * cs, rows)
        hi = min((r + 1) * cs, rows)
        out.append(hi - lo)
    return out


def chunk_offset(rows: int, world: int, rank: int) -> int:
    cs = (rows + world - 1) // world
    return min(rank * cs, rows)


def all_gather(tensors: Sequence[torch.Tensor], group: Optional[dist.ProcessGroup] = None) -> List[torch.Tensor]:
    """All-gather each tensor along dim 0 (equal local sizes), one bucketed collective per dtype.
    A DTensor (e.g. an FSDP2 gradient) is gathered to its full tensor over its own mesh."""
    tensors = list(tensors)
    if not is_available() or get_world_size(group) == 1 or not tensors:
        return tensors
    from .dtensor import is_dtensor

    if any(is_dtensor(t) for t in tensors):
        plain = [i for i, t in enumerate(tensors) if not is_dtensor(t)]
        out = [t.full_tensor() if is_dtensor(t) else None for t in tensors]
        for i, g in zip(plain, all_gather([tensors[i] for i in plain], group=group)):
            out[i] = g
        return out
    ws = get_world_size(group)
    out: List[Optional[torch.Tensor]] = [None] * len(tensors)
    buckets: "OrderedDict[tuple, List[int]]" = OrderedDict()
    for i, t in enumerate(tensors):
        buckets.setdefault((t.dtype, t.device), []).append(i)
    for (dtype, device), idxs in buckets.items():
        flat = [tensors[i].contiguous().reshape(-1) for i in idxs]
        sizes = [f.numel() for f in flat]
        send = torch.cat(flat) if len(flat) > 1 else flat[0]
        recv = send.new_empty(ws * send.numel())
        dist.all_gather_into_tensor(recv, send, group=group)
        recv = recv.view(ws, -1)
        off = 0
        for i, n in zip(idxs, sizes):
            t = tensors[i]
            parts = recv[:, off:off + n].reshape(ws, *t.shape)
            out[i] = parts.reshape(ws * t.shape[0], *t.shape[1:]) if t.dim() > 0 else parts.reshape(ws)
            off += n
    return out  # type: ignore[return-value]


def all_gather_grads(grads: Sequence[torch.Tensor], group: Optional[dist.ProcessGroup] = None) -> List[torch.Tensor]:
    """Gather row-sharded gradients into full matrices (``muon_fsdp.distributed.all_gather_grads``)."""
    return all_gather(grads, group=group)


def scatter(tensors: Sequence[torch.Tensor], src_rank: int = 0,
            group: Optional[dist.ProcessGroup] = None) -> List[torch.Tensor]:
    """Split each full tensor along dim 0 and give every rank its chunk (sent from ``src_rank``)."""
    tensors = list(tensors)
    if not is_available() or get_world_size(group) == 1:
        return tensors
    ws, rank = get_world_size(group), get_rank(group)
    out = []
    for t in tensors:
        t = t.contiguous()
        if t.shape[0] % ws != 0:
            raise ValueError(f"dim 0 ({t.shape[0]}) must be divisible by world_size ({ws}) for scatter")
        chunk = t.shape[0] // ws
        recv = t.new_empty((chunk,) + tuple(t.shape[1:]))
        src_global = dist.get_global_rank(group, src_rank) if group is not None else src_rank
        scatter_list = list(t.split(chunk)) if rank == src_rank else None
        dist.scatter(recv, scatter_list=scatter_list, src=src_global, group=group)
        out.append(recv)
    return out


def scatter_updates(updates: Sequence[torch.Tensor], src_rank: int = 0,
                    group: Optional[dist.ProcessGroup] = None) -> List[torch.Tensor]:
    """Each rank's ``torch.chunk`` row slice of identical full updates (no communication)."""
    updates = list(updates)
    if not is_available() or get_world_size(group) == 1:
        return updates
    ws, rank = get_world_size(group), get_rank(group)
    out = []
    for u in updates:
        rows = u.shape[0]
        off = chunk_offset(rows, ws, rank)
        n = chunk_rows(rows, ws)[rank]
        out.append(u[off:off + n].contiguous())
    return out


def _each(tensors):
    """A list of tensors (the reference's form) or one tensor (accepted as well)."""
    return [tensors] if isinstance(tensors, torch.Tensor) else list(tensors)


def all_reduce(tensors, op=None, group: Optional[dist.ProcessGroup] = None):
    """In-place all-reduce of each tensor (``op`` defaults to SUM); returns ``tensors``
    (``src/fsdp2_utils/comm.py:180-201``: a list of tensors; a single tensor also works)."""
    if not is_available() or get_world_size(group) == 1:
        return tensors
    for t in _each(tensors):
        dist.all_reduce(t, op=op if op is not None else dist.ReduceOp.SUM, group=group)
    return tensors


def all_reduce_sum(tensors, group: Optional[dist.ProcessGroup] = None):
    return all_reduce(tensors, dist.ReduceOp.SUM if is_available() else None, group)


def all_reduce_avg(tensors, group: Optional[dist.ProcessGroup] = None):
    """Sum, then divide by the group size (as the reference does, for every backend)."""
    if not is_available() or get_world_size(group) == 1:
        return tensors
    all_reduce(tensors, dist.ReduceOp.SUM, group)
    ws = get_world_size(group)
    for t in _each(tensors):
        t.div_(ws)
    return tensors


def broadcast(tensors, src_rank: int = 0, group: Optional[dist.ProcessGroup] = None, *, src: Optional[int] = None):
    """In-place broadcast of each tensor from ``src_rank`` (``src`` is accepted as an alias)."""
    if src is not None:
        src_rank = src
    if not is_available() or get_world_size(group) == 1:
        return tensors
    for t in _each(tensors):
        dist.broadcast(t, src=src_rank, group=group)
    return tensors


def barrier(group: Optional[dist.ProcessGroup] = None) -> None:
    if is_available():
        dist.barrier(group=group)


__all__ = [
    "is_available", "is_distributed", "get_world_size", "get_rank", "get_local_rank", "chunk_rows",
    "chunk_offset", "all_gather", "all_gather_grads", "scatter", "scatter_updates", "all_reduce",
    "all_reduce_sum", "all_reduce_avg", "broadcast", "barrier",
]
