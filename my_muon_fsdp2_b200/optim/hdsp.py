"""Hybrid-sharded (HSDP) Muon optimizer (parity: ``src/muon_fsdp/hdsp.py:142-486``).

Gradients are combined only inside the FSDP shard group (intra-node); replicas stay identical
because FSDP2's HSDP already all-reduced the gradients across the replicate dimension.  Math
per parameter (the reference's): a per-parameter accumulation gate on ``accum_count``, EMA
momentum ``buf = mu*buf + (1-mu)*g``, Nesterov ``g + mu*buf``, decoupled weight decay on >1-D
parameters, and for 2-D parameters ``p -= lr * sqrt(max/min) * ns_stepsize * NS(u)`` (the HSDP
variant's own dimension scale, hdsp.py:380-382); 1-D parameters ``p -= lr * u``.

Unlike the reference (whose step always raises: no ``@torch.no_grad``, hdsp.py:317), this runs,
and the NS work is split across the shard group by the owner-computes engine.
"""
from __future__ import annotations

import copy
import logging
from contextlib import contextmanager
from typing import Any, Dict, Iterator, List, Optional

import torch
import torch.nn as nn
from torch.optim import Optimizer

from ..ops.newton_schulz import hsdp_lr_scale
from ..parallel.fsdp_utils import collect_fsdp_modules
from ..parallel.mesh import create_device_mesh_2d, get_hsdp_groups
from ..parallel.muon_engine import MODE_EMA, MuonEngine, MuonHyper, MuonTask
from ._common import index_state_dict, load_index_state_dict, local_of, zeros_state_like

logger = logging.getLogger(__name__)


class HDSPMuonOptimizer(Optimizer):
    def __init__(self, model: nn.Module, device_mesh: Optional[Any] = None, dp_group: Optional[Any] = None,
                 fsdp_group: Optional[Any] = None, params: Optional[List[torch.nn.Parameter]] = None,
                 lr: float = 0.02, weight_decay: float = 0.01, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, ns_stepsize: float = 1.0, beta2: float = 0.99, eps: float = 1e-8,
                 gradient_accumulation_steps: int = 1, dp_size: Optional[int] = None,
                 fsdp_size: Optional[int] = None, comm: str = "auto"):
        self.model = model
        self.gradient_accumulation_steps = gradient_accumulation_steps
        self._step_count = 0
        if device_mesh is None:
            device_mesh = self._detect_device_mesh(model)
        if device_mesh is None and dp_size is not None and fsdp_size is not None:
            device_mesh = create_device_mesh_2d(dp_size, fsdp_size)
        self.device_mesh = device_mesh
        if device_mesh is not None:
            dpg, fg = get_hsdp_groups(device_mesh)
            dp_group = dp_group if dp_group is not None else dpg
            fsdp_group = fsdp_group if fsdp_group is not None else fg
        self.dp_group, self.fsdp_group = dp_group, fsdp_group
        if params is None:
            params = list(model.parameters())
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("HDSPMuonOptimizer received an empty parameter list")
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                        ns_stepsize=ns_stepsize, beta2=beta2, eps=eps)
        super().__init__(params, defaults)
        self._engine = MuonEngine(process_group=fsdp_group, comm=comm)
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state[p]
                st["momentum_buffer"] = zeros_state_like(p)
                st["second_moment"] = torch.zeros(0, device=local_of(p).device)
                st["accum_count"] = 0

    @staticmethod
    def _detect_device_mesh(model: nn.Module) -> Optional[Any]:
        """The 2-D mesh of the first FSDP2-sharded (DTensor) parameter, if any."""
        from ..parallel.dtensor import is_dtensor

        for p in model.parameters():
            if is_dtensor(p) and p.device_mesh.ndim == 2:
                return p.device_mesh
        return None

    @contextmanager
    def unshard_params(self) -> Iterator[None]:
        mods = collect_fsdp_modules(self.model)
        try:
            for m in mods:
                h = m.unshard(async_op=True)
                if h is not None:
                    h.wait()
            yield
        finally:
            for m in mods:
                try:
                    m.reshard()
                except Exception as e:  # pragma: no cover
                    logger.warning(f"reshard failed: {e}")

    @torch.no_grad()
    def step(self, closure: Any = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step_count += 1
        for group in self.param_groups:
            lr, wd = group["lr"], group["weight_decay"]
            tasks = []
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                st["accum_count"] = st.get("accum_count", 0) + 1
                if st["accum_count"] < self.gradient_accumulation_steps:
                    continue
                st["accum_count"] = 0
                is_mat = p.dim() > 1
                decay = (1.0 - lr * wd) if (wd > 0 and is_mat) else 1.0
                lr_eff = lr * hsdp_lr_scale(p.shape) * group["ns_stepsize"] if p.dim() == 2 else lr
                tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(st["momentum_buffer"]), lr_eff=lr_eff,
                                      decay=decay, orthogonalize=p.dim() == 2))
            hp = MuonHyper(mode=MODE_EMA, momentum=group["momentum"], nesterov=group["nesterov"] and
                           group["momentum"] > 0, ns_steps=group["ns_steps"])
            self._engine.step(tasks, hp)
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.detach_()
                    p.grad.zero_()

    def state_dict(self, include_state: bool = False) -> Dict[str, Any]:
        """``{"step_count", "param_groups"}`` with emptied ``params`` lists (the reference layout,
        hdsp.py:411-422, without mutating the live groups); ``include_state=True`` adds the
        momentum state in the standard indexed layout."""
        groups = []
        for g in self.param_groups:
            c = {k: copy.deepcopy(v) for k, v in g.items() if k != "params"}
            c["params"] = []
            groups.append(c)
        out: Dict[str, Any] = {"step_count": self._step_count, "param_groups": groups}
        if include_state:
            full = index_state_dict(self)
            out["state"] = full["state"]
            out["param_index_groups"] = [g["params"] for g in full["param_groups"]]
        return out

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        self._step_count = state_dict.get("step_count", 0)
        for g, sg in zip(self.param_groups, state_dict.get("param_groups", [])):
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
        if "state" in state_dict:
            idx_groups = state_dict.get("param_index_groups")
            groups = [dict(sg, params=ids) for sg, ids in zip(state_dict["param_groups"], idx_groups)]
            load_index_state_dict(self, {"state": state_dict["state"], "param_groups": groups})


class HSDPConfig:
    """HSDP configuration (hdsp.py:430-486)."""

    def __init__(self, dp_size: int = 1, fsdp_size: int = 1, lr: float = 0.02, momentum: float = 0.95,
                 weight_decay: float = 0.01, ns_steps: int = 5, nesterov: bool = True):
        self.dp_size, self.fsdp_size = dp_size, fsdp_size
        self.lr, self.momentum, self.weight_decay = lr, momentum, weight_decay
        self.ns_steps, self.nesterov = ns_steps, nesterov

    def create_device_mesh(self) -> Optional[Any]:
        return create_device_mesh_2d(self.dp_size, self.fsdp_size)

    def to_dict(self) -> Dict[str, Any]:
        return {"dp_size": self.dp_size, "fsdp_size": self.fsdp_size, "lr": self.lr, "momentum": self.momentum,
                "weight_decay": self.weight_decay, "ns_steps": self.ns_steps, "nesterov": self.nesterov}
