"""FSDP2-aware Muon optimizer (parity: ``src/muon_fsdp/fsdp.py:113-586``).

Constructor, defaults, state keys (``momentum_buffer``, ``second_moment``, ``accum_count``), the
``step_count`` checkpoint entry, ``unshard_params()``, ``zero_grad(set_to_none=False)`` and
``create_fsdp_muon_optimizer`` follow the reference.

``update_rule`` selects the math:

* ``"muon"`` (default) — the Muon update of ``MuonOptimizer`` (optimizer.py:102-172) with step
  ``lr * ns_stepsize``: EMA momentum, Nesterov, NS on 2-D parameters, decoupled weight decay.
  This is what the reference *intends*; its own step crashes under FSDP2 (fsdp.py:335 adds a
  local tensor to a DTensor buffer) and, on plain modules, discards the momentum result
  (fsdp.py:485) and never uses ``lr`` or ``weight_decay``.
* ``"reference"`` — the reference's literal behaviour on plain modules, for bit-level
  comparisons: the momentum / second-moment state is updated and discarded, and the applied
  update is ``p += -ns_stepsize * NS(grad)`` (NS skipped for 1-D: ``-ns_stepsize * grad``).

``second_moment`` is only allocated (full size) for ``update_rule="reference"``; under the
Muon rule it is a 0-element placeholder so that checkpoints keep the reference's key layout
without 4 bytes/parameter of dead state.
"""
from __future__ import annotations

import logging
from contextlib import contextmanager
from typing import Any, Dict, Iterator, List, Optional

import torch
import torch.nn as nn
from torch.optim import Optimizer

from ..ops.newton_schulz import muon_lr_scale, zeropower_via_newtonschulz5
from ..parallel.dtensor import get_local_tensor, is_dtensor
from ..parallel.fsdp_utils import collect_fsdp_modules
from ..parallel.muon_engine import MODE_EMA, MuonHyper, MuonTask
from ._common import default_engine, index_state_dict, load_index_state_dict, local_of, zeros_state_like
from .errors import InvalidParameterError

logger = logging.getLogger(__name__)


def _reference_moments(state, params, mu: float, wd: float, beta2: float, nesterov: bool) -> None:
    """Momentum and second-moment state of the reference update rule (fsdp.py:326-345):
    g = grad + wd p, buf = mu buf + g, u = g + mu buf (Nesterov) or buf, sm = beta2 sm + (1-beta2) u^2.
    On CUDA one ``muon_moments`` launch per (param dtype, grad dtype) bucket reads each tensor once;
    elsewhere the same steps as PyTorch ops."""
    live = [p for p in params if p.grad is not None]
    if not live:
        return
    locs = [(get_local_tensor(p), get_local_tensor(p.grad), local_of(state[p]["momentum_buffer"]),
             local_of(state[p]["second_moment"])) for p in live]
    if locs[0][0].is_cuda:
        from .._ext import ext

        buckets: Dict[Any, List[int]] = {}
        for i, (pd, gd, _, _) in enumerate(locs):
            buckets.setdefault((pd.dtype, gd.dtype), []).append(i)
        for idx in buckets.values():
            ext().muon_moments([locs[i][0].contiguous() for i in idx], [locs[i][1].contiguous() for i in idx],
                               [locs[i][2] for i in idx], [locs[i][3] for i in idx], mu, beta2, wd, nesterov)
        return
    for pd, gd, buf, sm in locs:
        g = gd + wd * pd if wd != 0 else gd
        buf.mul_(mu).add_(g.to(buf.dtype))
        g = g + mu * buf if nesterov else buf.clone()
        sm.mul_(beta2).addcmul_(g, g, value=1 - beta2)


class FSDPMuonOptimizer(Optimizer):
    def __init__(
        self,
        model: nn.Module,
        params: Optional[List[torch.nn.Parameter]] = None,
        lr: float = 0.02,
        weight_decay: float = 0.01,
        momentum: float = 0.95,
        nesterov: bool = True,
        ns_steps: int = 5,
        ns_stepsize: float = 1.0,
        beta2: float = 0.99,
        eps: float = 1e-8,
        gradient_accumulation_steps: int = 1,
        *,
        update_rule: str = "muon",
        process_group=None,
        comm: str = "auto",
    ):
        if update_rule not in ("muon", "reference"):
            raise ValueError(f"update_rule must be 'muon' or 'reference', got {update_rule!r}")
        if gradient_accumulation_steps < 1:
            raise InvalidParameterError(f"Invalid gradient_accumulation_steps: {gradient_accumulation_steps}")
        self.model = model
        self.gradient_accumulation_steps = gradient_accumulation_steps
        self.update_rule = update_rule
        self._step_count = 0
        if params is None:
            params = list(model.parameters())
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("FSDPMuonOptimizer received an empty parameter list")
        self.fsdp_modules = collect_fsdp_modules(model)
        if self.fsdp_modules:
            logger.info(f"found {len(self.fsdp_modules)} FSDP2 modules")
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                        ns_stepsize=ns_stepsize, beta2=beta2, eps=eps)
        super().__init__(params, defaults)
        self._engine = default_engine(process_group, comm)
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state[p]
                st["momentum_buffer"] = zeros_state_like(p)
                if update_rule == "reference":
                    st["second_moment"] = zeros_state_like(p)
                else:
                    st["second_moment"] = torch.zeros(0, dtype=torch.float32, device=get_local_tensor(p).device)
                st["accum_count"] = 0

    @contextmanager
    def unshard_params(self) -> Iterator[None]:
        """Unshard every FSDP2 module inside the block; always reshard on exit (fsdp.py:216-251)."""
        if not self.fsdp_modules:
            yield
            return
        handles = []
        try:
            for m in self.fsdp_modules:
                h = m.unshard(async_op=True)
                handles.append(m)
                if h is not None:
                    h.wait()
            yield
        finally:
            for m in handles:
                try:
                    m.reshard()
                except Exception as e:  # pragma: no cover
                    logger.warning(f"reshard failed: {e}")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step_count += 1
        for group in self.param_groups:
            for p in group["params"]:
                self.state[p]["accum_count"] = self._step_count % self.gradient_accumulation_steps
        if self._step_count % self.gradient_accumulation_steps != 0:
            return loss
        for group in self.param_groups:
            if self.update_rule == "reference":
                self._reference_group(group)
            else:
                self._muon_group(group)
        return loss

    def _muon_group(self, group: Dict[str, Any]) -> None:
        lr, wd, step = group["lr"], group["weight_decay"], group["ns_stepsize"]
        tasks = []
        for p in group["params"]:
            if p.grad is None:
                continue
            is2d = p.dim() == 2
            scale = muon_lr_scale(p.shape) if is2d else 1.0
            tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(self.state[p]["momentum_buffer"]),
                                  lr_eff=lr * step * scale, decay=1.0 - lr * wd, orthogonalize=is2d))
        hp = MuonHyper(mode=MODE_EMA, momentum=group["momentum"], nesterov=group["nesterov"],
                       ns_steps=group["ns_steps"])
        self._engine.step(tasks, hp)

    def _reference_group(self, group: Dict[str, Any]) -> None:
        """Literal fsdp.py:294-450 on local tensors (the state update is computed and discarded)."""
        from ..parallel.comm import all_gather_grads, chunk_offset, chunk_rows, get_rank, get_world_size

        mu, wd, beta2, eps, lr = group["momentum"], group["weight_decay"], group["beta2"], group["eps"], group["lr"]
        params = group["params"]
        _reference_moments(self.state, params, mu, wd, beta2, group["nesterov"])
        grads = [get_local_tensor(p.grad) if p.grad is not None else torch.zeros_like(get_local_tensor(p))
                 for p in params]
        ws = get_world_size()
        gathered = all_gather_grads(grads) if ws > 1 else grads
        rank = get_rank()
        for p, g in zip(params, gathered):
            if p.grad is None:
                continue
            if g.dim() < 2:
                u = -g * group["ns_stepsize"]
            else:
                u = -zeropower_via_newtonschulz5(g.reshape(g.shape[0], -1), steps=group["ns_steps"]).reshape(
                    g.shape) * group["ns_stepsize"]
            pd = get_local_tensor(p)
            if ws > 1 and is_dtensor(p):
                off = chunk_offset(u.shape[0], ws, rank)
                u = u[off:off + chunk_rows(u.shape[0], ws)[rank]]
            pd.add_(u.reshape(pd.shape).to(pd.dtype))

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
        """``{"state", "param_groups", "step_count"}`` with the reference's per-parameter keys."""
        return index_state_dict(self, {"step_count": self._step_count})

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        self._step_count = state_dict.get("step_count", 0)
        load_index_state_dict(self, state_dict)


def create_fsdp_muon_optimizer(
    model: nn.Module,
    lr: float = 0.02,
    weight_decay: float = 0.01,
    momentum: float = 0.95,
    nesterov: bool = True,
    ns_steps: int = 5,
    ns_stepsize: float = 1.0,
    beta2: float = 0.99,
    eps: float = 1e-8,
    gradient_accumulation_steps: int = 1,
    **kwargs,
) -> FSDPMuonOptimizer:
    """Convenience constructor (fsdp.py:544-586)."""
    return FSDPMuonOptimizer(model=model, lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                             ns_steps=ns_steps, ns_stepsize=ns_stepsize, beta2=beta2, eps=eps,
                             gradient_accumulation_steps=gradient_accumulation_steps, **kwargs)
