"""Model-first Muon optimizer of the ``fsdp2_utils`` API (parity: ``src/fsdp2_utils/muon.py:14-144``).

Math: coupled weight decay ``g <- g + wd * p``, EMA momentum, Nesterov ``g + mu * buf``,
NS on 2-D parameters with the (unit) dimension scale, ``p -= lr * u``.

Unlike the reference, the momentum buffer persists across steps (the reference rebuilds it
whenever the gathered gradient shape differs from the buffer, muon.py:113-114, and never stores
it back) and weight decay works on sharded parameters (muon.py:121 crashes there): everything
runs on local shards through the owner-computes engine.
"""
from __future__ import annotations

from typing import List, Optional

import torch.nn as nn

from ..ops.newton_schulz import muon_lr_scale
from ..parallel.muon_engine import MODE_EMA, MuonHyper, MuonTask
from ._common import default_engine, local_of, zeros_state_like
from .base import FSDPCompatibleOptimizer
from .muon import _validate


class MuonOptimizer(FSDPCompatibleOptimizer):
    def __init__(self, model: nn.Module, params: Optional[List[nn.Parameter]] = None, lr: float = 0.02,
                 momentum: float = 0.95, weight_decay: float = 0.0, nesterov: bool = False, ns_steps: int = 5,
                 gradient_accumulation_steps: int = 1, *, process_group=None, comm: str = "auto") -> None:
        _validate(lr, momentum, weight_decay, ns_steps, nesterov)
        defaults = dict(lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=nesterov, ns_steps=ns_steps)
        super().__init__(model=model, params=params, defaults=defaults,
                         gradient_accumulation_steps=gradient_accumulation_steps)
        self._engine = default_engine(process_group, comm)
        for group in self.param_groups:
            for p in group["params"]:
                self.state[p]["momentum_buffer"] = zeros_state_like(p)

    def _step_impl(self) -> None:
        for group in self.param_groups:
            lr = group["lr"]
            tasks = []
            for p in group["params"]:
                if p.grad is None:
                    continue
                is2d = p.dim() == 2
                scale = muon_lr_scale(p.shape) if is2d else 1.0
                tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(self.state[p]["momentum_buffer"]),
                                      lr_eff=lr * scale, decay=1.0, orthogonalize=is2d))
            hp = MuonHyper(mode=MODE_EMA, momentum=group["momentum"], nesterov=group["nesterov"],
                           wd_coupled=group["weight_decay"], ns_steps=group["ns_steps"])
            self._engine.step(tasks, hp)


__all__ = ["MuonOptimizer"]
