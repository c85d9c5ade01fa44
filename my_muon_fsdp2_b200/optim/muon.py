"""Single-entry Muon optimizer (parity: ``src/muon_fsdp/optimizer.py:15-190``).

Math per parameter (the reference's, unchanged)::

    buf = lerp(buf, g, 1 - momentum)                  # EMA
    u   = g + momentum * buf  if nesterov else buf
    if p is 2-D:  u = NS5(u) * max(1, min/max)**0.5   # the scale is always 1.0
    p  *= 1 - lr * weight_decay                       # decoupled, all params
    p  -= lr * u

Execution: CUDA parameters go through :class:`~my_muon_fsdp2_b200.parallel.muon_engine.MuonEngine`
(one fused momentum kernel per group, one batched tcgen05 NS chain per shape, the update fused
into the last GEMM epilogue).  FSDP2 DTensor parameters are handled natively (owner-computes NS,
no redundant work) instead of through DTensor op dispatch.  CPU parameters run the same math
with PyTorch ops.
"""
from __future__ import annotations

from typing import Any, Callable, Optional

import torch
from torch.optim.optimizer import Optimizer

from ..ops.newton_schulz import muon_lr_scale
from ..parallel.muon_engine import MODE_EMA, MuonHyper, MuonTask
from ._common import default_engine, load_index_state_dict, local_of, zeros_state_like
from .errors import InvalidParameterError, SparseGradientError


def _validate(lr, momentum, weight_decay, ns_steps, nesterov):
    if lr < 0.0:
        raise InvalidParameterError(f"Invalid learning rate: {lr}")
    if momentum < 0.0 or momentum > 1.0:
        raise InvalidParameterError(f"Invalid momentum value: {momentum}")
    if weight_decay < 0.0:
        raise InvalidParameterError(f"Invalid weight_decay value: {weight_decay}")
    if ns_steps < 0:
        raise InvalidParameterError(f"Invalid ns_steps value: {ns_steps}")
    if nesterov and momentum <= 0:
        raise InvalidParameterError("Nesterov momentum requires a positive momentum")


class MuonOptimizer(Optimizer):
    """Muon with momentum, Newton–Schulz orthogonalisation of 2-D updates and weight decay.

    Args:
        params: iterable of parameters or parameter-group dicts.
        lr: learning rate (0.02).  momentum: EMA coefficient (0.95).
        weight_decay: decoupled weight decay (0).  nesterov: Nesterov form (False).
        ns_steps: Newton–Schulz iterations (5).
        process_group / comm: optional overrides for the sharded engine.
        schedule: "auto" picks owner-computes or the cooperative all-rank chain per matrix shape
            (``select_split``); "never" / "always" force one of them (eligible shapes only).
    """

    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, weight_decay: float = 0.0,
                 nesterov: bool = False, ns_steps: int = 5, *, process_group=None, comm: str = "auto",
                 schedule: str = "auto") -> None:
        _validate(lr, momentum, weight_decay, ns_steps, nesterov)
        defaults = dict(lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=nesterov, ns_steps=ns_steps)
        super().__init__(params, defaults)
        self._engine = default_engine(process_group, comm, schedule)

    def __setstate__(self, state: dict) -> None:
        super().__setstate__(state)
        for group in self.param_groups:
            group.setdefault("nesterov", False)
        if not hasattr(self, "_engine"):
            self._engine = default_engine()

    @torch.no_grad()
    def step(self, closure: Optional[Callable[[], Any]] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, wd = group["lr"], group["weight_decay"]
            tasks = []
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise SparseGradientError("MuonOptimizer does not support sparse gradients")
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = zeros_state_like(p)
                is2d = p.dim() == 2
                scale = muon_lr_scale(p.shape) if is2d else 1.0
                tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(st["momentum_buffer"]), lr_eff=lr * scale,
                                      decay=1.0 - lr * wd, orthogonalize=is2d))
            hp = MuonHyper(mode=MODE_EMA, momentum=group["momentum"], nesterov=group["nesterov"],
                           ns_steps=group["ns_steps"])
            self._engine.step(tasks, hp)
        return loss

    def state_dict(self) -> dict:
        return super().state_dict()

    def load_state_dict(self, state_dict: dict) -> None:
        # torch.optim would cast the fp32 momentum to the (bf16) parameter dtype; keep fp32.
        load_index_state_dict(self, state_dict)
