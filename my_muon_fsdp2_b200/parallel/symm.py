"""Symmetric-memory workspace for in-kernel NVLink exchange (P2P loads/stores).

One bf16 buffer per process group, allocated with ``torch.distributed._symmetric_memory`` and
mapped into every peer.  The Muon engine uses it *in place*: each rank's momentum kernel writes
the NS input of its row shard of matrix *j* at a fixed offset, the owner's assembly kernel reads
those shards straight from the peers (P2P loads), and the owner's final GEMM epilogue writes
every rank's row shard of the result back into the same region of that rank (P2P stores).
Ordering between the phases uses :meth:`barrier`, a one-block kernel over the signal pads with
bounded waits (``csrc/symm_comm.cu``), which can also deliver a small fp32 payload row to every
peer (the per-matrix partial sums of squares).
"""
from __future__ import annotations

import weakref
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


class SymmWorkspace:
    def __init__(self, group: dist.ProcessGroup, device: torch.device, timeout_s: float = 30.0):
        import torch.distributed._symmetric_memory as symm_mem

        self._sm = symm_mem
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self.buf: Optional[torch.Tensor] = None
        self.handle = None
        self.payload: Optional[torch.Tensor] = None
        self.payload_handle = None
        self.epoch = 0

    def _rdv(self, t: torch.Tensor):
        try:
            return self._sm.rendezvous(t, self.group)
        except TypeError:
            return self._sm.rendezvous(t, self.group.group_name)

    def ensure(self, numel: int, n_payload: int) -> None:
        """Collective: (re)allocate so that the buffer holds ``numel`` bf16 and the payload
        ``world * n_payload`` fp32.  Every rank must call it with the same arguments."""
        numel = max(int(numel), 1)
        n_payload = max(int(n_payload), 1)
        if self.buf is None or self.buf.numel() < numel:
            cap = max(numel, int(1.25 * (self.buf.numel() if self.buf is not None else 0)))
            self.buf = self._sm.empty(cap, dtype=torch.bfloat16, device=self.device)
            self.handle = self._rdv(self.buf)
            self.buf_ptrs = list(self.handle.buffer_ptrs)
            self.pad_ptrs = torch.tensor(list(self.handle.signal_pad_ptrs), dtype=torch.int64, device=self.device)
            self.epoch = 0
        if self.payload is None or self.payload.numel() < self.world * n_payload:
            self.payload = self._sm.empty(self.world * n_payload, dtype=torch.float32, device=self.device)
            self.payload_handle = self._rdv(self.payload)
            self.payload_ptrs = torch.tensor(list(self.payload_handle.buffer_ptrs), dtype=torch.int64,
                                             device=self.device)
        self.n_payload = n_payload

    def peer_view(self, peer: int, offset: int, shape) -> torch.Tensor:
        """Tensor view of ``shape`` bf16 elements at ``offset`` in ``peer``'s buffer."""
        if peer == self.rank:
            n = 1
            for s in shape:
                n *= s
            return self.buf[offset:offset + n].view(*shape)
        return self.handle.get_buffer(peer, tuple(shape), torch.bfloat16, offset)

    def peer_addr(self, peer: int, offset: int) -> int:
        return int(self.buf_ptrs[peer]) + 2 * int(offset)

    def barrier(self, payload: Optional[torch.Tensor] = None) -> None:
        from .._ext import ext

        self.epoch += 1
        if payload is not None:
            assert payload.numel() == self.n_payload
            ext().symm_barrier(self.pad_ptrs, self.rank, self.world, self.epoch, 0, payload.contiguous(),
                               self.payload_ptrs, self.timeout_s)
        else:
            ext().symm_barrier(self.pad_ptrs, self.rank, self.world, self.epoch, 0, None, None, self.timeout_s)

    def payload_rows(self) -> torch.Tensor:
        return self.payload[: self.world * self.n_payload].view(self.world, self.n_payload)


_WORKSPACES: Dict[int, SymmWorkspace] = {}

# Peer-mapped storage that holds parameters (the shard buffers of the fused FSDP linears):
# (weak reference to the buffer, ranks of its group, each rank's base address).  The Muon
# engine's final epilogue writes a parameter's update straight into every rank's shard of it
# when the parameter lives here.
_PEER_STORES: List[Tuple["weakref.ref", Tuple[int, ...], List[int]]] = []


def register_peer_storage(buf: torch.Tensor, group: dist.ProcessGroup, buffer_ptrs: Sequence[int]) -> None:
    """Record a symmetric buffer (same layout on every rank of ``group``) whose views are
    parameters; ``buffer_ptrs[r]`` is rank r's copy as mapped into this process."""
    ranks = tuple(dist.get_process_group_ranks(group))
    _PEER_STORES[:] = [e for e in _PEER_STORES if e[0]() is not None]
    _PEER_STORES.append((weakref.ref(buf), ranks, [int(x) for x in buffer_ptrs]))


def peer_param_addrs(t: torch.Tensor, group: dist.ProcessGroup) -> Optional[List[int]]:
    """Address of ``t``'s first element in every rank's copy of the registered symmetric
    buffer that holds it (the same offset on every rank), or None when ``t`` is not in
    peer-mapped storage of ``group``'s ranks."""
    if not t.is_contiguous():
        return None
    ptr = t.data_ptr()
    ranks = None
    for ref, rk, bases in _PEER_STORES:
        buf = ref()
        if buf is None or buf.device != t.device:
            continue
        lo = buf.data_ptr()
        if lo <= ptr and ptr + t.numel() * t.element_size() <= lo + buf.numel() * buf.element_size():
            if ranks is None:
                ranks = tuple(dist.get_process_group_ranks(group))
            if rk != ranks:
                return None
            return [b + (ptr - lo) for b in bases]
    return None


def workspace_for(group: dist.ProcessGroup, device: torch.device) -> SymmWorkspace:
    key = id(group)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = SymmWorkspace(group, device)
        _WORKSPACES[key] = ws
    return ws


def p2p_supported(group: dist.ProcessGroup) -> bool:
    """Symmetric memory needs CUDA tensors, NCCL, and the extension."""
    try:
        return dist.get_backend(group) == "nccl" and torch.cuda.is_available()
    except Exception:
        return False
