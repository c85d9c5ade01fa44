"""FSDP2 module helpers (parity: ``src/fsdp2_utils/fsdp_utils.py`` and ``src/muon_fsdp/fsdp.py:74-110``).

``HAS_FSDP2`` only needs ``fully_shard``/``FSDPModule`` (the reference additionally imports
FSDP1-only names, fsdp_utils.py:19-26).
"""
from __future__ import annotations

import logging
from contextlib import contextmanager
from typing import Iterator, List, Optional

import torch
import torch.nn as nn

from .dtensor import get_local_tensor

logger = logging.getLogger(__name__)

try:
    from torch.distributed.fsdp import FSDPModule, fully_shard  # noqa: F401

    HAS_FSDP2 = True
except ImportError:  # pragma: no cover
    FSDPModule = None  # type: ignore
    HAS_FSDP2 = False


def is_fsdp_module(module: nn.Module) -> bool:
    return HAS_FSDP2 and isinstance(module, FSDPModule)


def collect_fsdp_modules(model: nn.Module) -> List[nn.Module]:
    if not HAS_FSDP2:
        logger.warning("FSDP2 is not available; running single-process")
        return []
    return [m for m in model.modules() if isinstance(m, FSDPModule)]


def has_fsdp_modules(model: nn.Module) -> bool:
    return len(collect_fsdp_modules(model)) > 0


@contextmanager
def unshard_modules(modules: List[nn.Module]) -> Iterator[None]:
    """Unshard every FSDP2 module for the duration of the block; always reshard on exit."""
    mods = [m for m in modules if is_fsdp_module(m)]
    handles = []
    try:
        for m in mods:
            h = m.unshard(async_op=True)
            handles.append((m, h))
        for _, h in handles:
            if h is not None:
                h.wait()
        yield
    finally:
        for m, _ in handles:
            try:
                m.reshard()
            except Exception as e:  # pragma: no cover
                logger.warning(f"reshard failed: {e}")


@contextmanager
def unshard_model(model: nn.Module) -> Iterator[None]:
    with unshard_modules(collect_fsdp_modules(model)):
        yield


def get_model_params_with_grad(model: nn.Module) -> List[nn.Parameter]:
    return [p for p in model.parameters() if p.requires_grad]


def get_local_params(params: List[nn.Parameter]) -> List[torch.Tensor]:
    return [get_local_tensor(p) for p in params]


def get_local_grads(params: List[nn.Parameter]) -> List[Optional[torch.Tensor]]:
    return [None if p.grad is None else get_local_tensor(p.grad) for p in params]


@torch.no_grad()
def apply_local_updates(params: List[nn.Parameter], updates: List[Optional[torch.Tensor]]) -> None:
    for p, u in zip(params, updates):
        if u is None:
            continue
        lp = get_local_tensor(p)
        lp.add_(u.reshape(lp.shape).to(lp.dtype))


__all__ = ["HAS_FSDP2", "is_fsdp_module", "collect_fsdp_modules", "has_fsdp_modules", "unshard_modules",
           "unshard_model", "get_model_params_with_grad", "get_local_params", "get_local_grads",
           "apply_local_updates"]
