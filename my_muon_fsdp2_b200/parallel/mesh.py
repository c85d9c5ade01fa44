"""2-D (replicate x shard) device meshes for HSDP.

Parity: ``create_device_mesh_2d``, ``get_hsdp_groups`` and ``gather_grads_group`` of
``src/muon_fsdp/hdsp.py:49-139``.  The mesh really is ``(dp_size, fsdp_size)`` with dims
``("dp_replicate", "fsdp_shard")`` (the reference builds ``(1, dp*fsdp)``, hdsp.py:76-80), and
``gather_grads_group`` raises on a failed collective instead of silently returning the local
gradients (hdsp.py:137-139) unless ``fallback_on_error=True``.
"""
from __future__ import annotations

import logging
from typing import Any, List, Optional, Tuple

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


def create_device_mesh_2d(dp_size: int, fsdp_size: int, device_type: Optional[str] = None) -> Optional[Any]:
    """``init_device_mesh(device, (dp_size, fsdp_size), ("dp_replicate", "fsdp_shard"))`` or None."""
    if not (dist.is_available() and dist.is_initialized()):
        return None
    if dp_size * fsdp_size != dist.get_world_size():
        raise ValueError(f"dp_size*fsdp_size ({dp_size}*{fsdp_size}) must equal world size {dist.get_world_size()}")
    from torch.distributed.device_mesh import init_device_mesh

    if device_type is None:
        device_type = "cuda" if torch.cuda.is_available() and dist.get_backend() == "nccl" else "cpu"
    return init_device_mesh(device_type, (dp_size, fsdp_size), mesh_dim_names=("dp_replicate", "fsdp_shard"))


def get_hsdp_groups(mesh: Any) -> Tuple[Optional[Any], Optional[Any]]:
    try:
        return mesh.get_group("dp_replicate"), mesh.get_group("fsdp_shard")
    except Exception:
        return None, None


def gather_grads_group(grads: List[torch.Tensor], group: Any, fallback_on_error: bool = False) -> List[torch.Tensor]:
    """All-gather each gradient along dim 0 inside ``group`` (one bucketed collective per dtype)."""
    if group is None or not (dist.is_available() and dist.is_initialized()):
        return grads
    if dist.get_world_size(group) == 1:
        return grads
    from .comm import all_gather

    try:
        return all_gather(grads, group=group)
    except Exception as e:
        if fallback_on_error:
            logger.warning(f"gather within group failed ({e}); using local gradients")
            return grads
        raise
