"""DTensor helpers (parity: ``src/fsdp2_utils/dtensor.py`` and ``src/muon_fsdp/fsdp.py:29-71``).

``redistribute_dtensor`` works here (the reference calls an undefined ``redistribute``,
dtensor.py:160).
"""
from __future__ import annotations

import logging
from typing import Any, Optional

import torch

logger = logging.getLogger(__name__)

try:
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.tensor import DTensor, Replicate, Shard, distribute_tensor

    HAS_DTENSOR = True
except ImportError:  # pragma: no cover
    HAS_DTENSOR = False
    DTensor = None  # type: ignore


def is_dtensor(tensor: Any) -> bool:
    return HAS_DTENSOR and isinstance(tensor, DTensor)


def get_local_tensor(tensor: torch.Tensor) -> torch.Tensor:
    return tensor.to_local() if is_dtensor(tensor) else tensor


def get_full_tensor(tensor: torch.Tensor) -> torch.Tensor:
    return tensor.full_tensor() if is_dtensor(tensor) else tensor


# muon_fsdp.fsdp names
get_dtensor_local_tensor = get_local_tensor
get_dtensor_full_tensor = get_full_tensor


def get_shard_dim(tensor: torch.Tensor) -> Optional[int]:
    if not is_dtensor(tensor):
        return None
    for p in tensor.placements:
        if isinstance(p, Shard):
            return p.dim
    return None


def create_dtensor(tensor: torch.Tensor, device_mesh: Optional["DeviceMesh"] = None, shard_dim: int = 0, *,
                   replicate: bool = False) -> torch.Tensor:
    if not HAS_DTENSOR:
        raise RuntimeError("DTensor is not available in this torch build")
    if device_mesh is None:
        import torch.distributed as dist

        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("create_dtensor needs an initialised process group or an explicit device_mesh")
        device_mesh = DeviceMesh(tensor.device.type, list(range(dist.get_world_size())))
    placement = Replicate() if replicate else Shard(shard_dim)
    return distribute_tensor(tensor, device_mesh, [placement])


def redistribute_dtensor(tensor: torch.Tensor, device_mesh: Optional["DeviceMesh"] = None,
                         shard_dim: Optional[int] = None, *, replicate: bool = False) -> torch.Tensor:
    if not is_dtensor(tensor):
        return tensor
    mesh = device_mesh if device_mesh is not None else tensor.device_mesh
    if replicate:
        placements = [Replicate()]
    elif shard_dim is not None:
        placements = [Shard(shard_dim)]
    else:
        placements = list(tensor.placements)
    if mesh is tensor.device_mesh:
        return tensor.redistribute(placements=placements)
    return distribute_tensor(tensor.full_tensor(), mesh, placements)


def dtensor_meta_info(tensor: torch.Tensor) -> dict:
    info = {"is_dtensor": False, "local_shape": tensor.shape, "global_shape": tensor.shape, "shard_dim": None,
            "device_mesh_shape": None}
    if is_dtensor(tensor):
        info.update(is_dtensor=True, local_shape=tensor.to_local().shape, shard_dim=get_shard_dim(tensor),
                    device_mesh_shape=tuple(tensor.device_mesh.shape))
    return info


__all__ = ["HAS_DTENSOR", "is_dtensor", "get_local_tensor", "get_full_tensor", "get_dtensor_local_tensor",
           "get_dtensor_full_tensor", "get_shard_dim", "create_dtensor", "redistribute_dtensor", "dtensor_meta_info"]
