"""FSDP2-compatible optimizer base class (parity: ``src/fsdp2_utils/base.py:32-238``).

Subclasses implement ``_step_impl``; ``step`` runs it only every
``gradient_accumulation_steps``-th call.  Helpers gather local gradient shards, hand back each
rank's slice of a full update and apply updates to the local shards.  ``state_dict`` carries
``step_count`` next to the usual ``state`` / ``param_groups``.
"""
from __future__ import annotations

import logging
from typing import Any, Callable, Dict, List, Optional

import torch
import torch.nn as nn
from torch.optim import Optimizer

from ..parallel.comm import all_gather_grads, get_world_size, is_distributed, scatter_updates
from ..parallel.dtensor import get_local_tensor, is_dtensor
from ..parallel.fsdp_utils import collect_fsdp_modules
from ._common import index_state_dict, load_index_state_dict
from .errors import InvalidParameterError

logger = logging.getLogger(__name__)


class FSDPCompatibleOptimizer(Optimizer):
    def __init__(self, model: nn.Module, params: Optional[List[nn.Parameter]] = None,
                 defaults: Optional[Dict[str, Any]] = None, gradient_accumulation_steps: int = 1) -> None:
        if gradient_accumulation_steps < 1:
            raise InvalidParameterError(f"Invalid gradient_accumulation_steps: {gradient_accumulation_steps}")
        self.model = model
        self.gradient_accumulation_steps = gradient_accumulation_steps
        self._step_count = 0
        if params is None:
            params = list(model.parameters())
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("optimizer received an empty parameter list")
        self.fsdp_modules = collect_fsdp_modules(model)
        super().__init__(params, defaults or {})

    @torch.no_grad()
    def step(self, closure: Optional[Callable[[], float]] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step_count += 1
        if self._step_count % self.gradient_accumulation_steps == 0:
            self._step_impl()
        return loss

    def _step_impl(self) -> None:
        raise NotImplementedError("subclasses must implement _step_impl")

    def _gather_gradients(self, params: List[nn.Parameter]) -> List[Optional[torch.Tensor]]:
        """Full gradients (all-gathered along dim 0 for sharded params); None where no grad."""
        local = [None if p.grad is None else (get_local_tensor(p.grad) if is_dtensor(p) else p.grad) for p in params]
        if is_distributed() and get_world_size() > 1:
            idx = [i for i, (p, g) in enumerate(zip(params, local)) if g is not None and is_dtensor(p)]
            if idx:
                full = all_gather_grads([local[i] for i in idx])
                for i, f in zip(idx, full):
                    local[i] = f[: params[i].shape[0]]
        return local

    def _scatter_updates(self, params: List[nn.Parameter], updates: List[Optional[torch.Tensor]]
                         ) -> List[Optional[torch.Tensor]]:
        """This rank's slice of each full update (sharded params) or the update itself."""
        if get_world_size() <= 1:
            return updates
        out: List[Optional[torch.Tensor]] = []
        for p, u in zip(params, updates):
            if u is None or not is_dtensor(p):
                out.append(u)
            else:
                out.append(scatter_updates([u])[0])
        return out

    def _apply_updates(self, params: List[nn.Parameter], updates: List[Optional[torch.Tensor]]) -> None:
        for p, u in zip(params, updates):
            if u is None:
                continue
            lp = get_local_tensor(p)
            lp.add_(u.reshape(lp.shape).to(lp.dtype))

    def zero_grad(self, set_to_none: bool = False) -> None:
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                if set_to_none:
                    p.grad = None
                else:
                    if p.grad.grad_fn is not None:
                        p.grad.detach_()
                    else:
                        p.grad.requires_grad_(False)
                    p.grad.zero_()

    def state_dict(self) -> Dict[str, Any]:
        return index_state_dict(self, {"step_count": self._step_count})

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        self._step_count = state_dict.get("step_count", 0)
        load_index_state_dict(self, state_dict)


__all__ = ["FSDPCompatibleOptimizer"]
