"""Spectral-Sphere optimizer (parity: ``src/muon_fsdp/sso.py:34-292``).

Per 2-D parameter: sigma by power iteration, target radius R (``spectral_mup`` / ``identity``),
retraction of the weight onto the sphere (``hard`` / ``dynamic``), then the Muon update (EMA
momentum, optional Nesterov, NS, decoupled weight decay).

On CUDA the retraction factor never leaves the device: it is folded into the per-matrix
``p_scale`` of the fused NS epilogue (``p <- (1 - lr*wd) * r * p - lr * O``), so the whole step
has no host synchronisation (the reference calls ``.item()`` twice per matrix per step).
``state["current_sigma"]`` is then a 0-dim device tensor; :meth:`get_spectral_norms` returns
floats as in the reference.
"""
from __future__ import annotations

from typing import Any, Optional

import torch
from torch.optim.optimizer import Optimizer

from ..ops.newton_schulz import muon_lr_scale
from ..ops.spectral import compute_target_radius, power_iteration, retraction_scale
from ..parallel.dtensor import is_dtensor
from ..parallel.muon_engine import MODE_EMA, MuonHyper, MuonTask
from ._common import default_engine, load_index_state_dict, local_of, zeros_state_like
from .errors import InvalidParameterError, SparseGradientError


class SpectralSphereOptimizer(Optimizer):
    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, weight_decay: float = 0.0,
                 nesterov: bool = False, ns_steps: int = 5, power_iteration_steps: int = 10,
                 radius_mode: str = "spectral_mup", radius_scaler: float = 1.0, retract_mode: str = "hard") -> None:
        if lr < 0.0:
            raise InvalidParameterError(f"Invalid learning rate: {lr}")
        if momentum < 0.0 or momentum > 1.0:
            raise InvalidParameterError(f"Invalid momentum value: {momentum}")
        if weight_decay < 0.0:
            raise InvalidParameterError(f"Invalid weight_decay value: {weight_decay}")
        if ns_steps < 0:
            raise InvalidParameterError(f"Invalid ns_steps value: {ns_steps}")
        if power_iteration_steps < 1:
            raise InvalidParameterError(f"Invalid power_iteration_steps value: {power_iteration_steps}")
        if nesterov and momentum <= 0:
            raise InvalidParameterError("Nesterov momentum requires positive momentum")
        if radius_mode not in ("spectral_mup", "identity"):
            raise InvalidParameterError(f"Invalid radius_mode: {radius_mode}")
        if retract_mode not in ("hard", "dynamic"):
            raise InvalidParameterError(f"Invalid retract_mode: {retract_mode}")
        defaults = dict(lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=nesterov, ns_steps=ns_steps,
                        power_iteration_steps=power_iteration_steps, radius_mode=radius_mode,
                        radius_scaler=radius_scaler, retract_mode=retract_mode)
        super().__init__(params, defaults)
        self._engine = default_engine()

    def __setstate__(self, state: dict) -> None:
        super().__setstate__(state)
        for g in self.param_groups:
            g.setdefault("nesterov", False)
            g.setdefault("power_iteration_steps", 10)
            g.setdefault("radius_mode", "spectral_mup")
            g.setdefault("radius_scaler", 1.0)
            g.setdefault("retract_mode", "hard")
        if not hasattr(self, "_engine"):
            self._engine = default_engine()

    @staticmethod
    def _sigma(p: torch.Tensor, iters: int):
        w = p.full_tensor() if is_dtensor(p) else p
        sigma, _, _ = power_iteration(w.detach(), num_iterations=iters)
        return sigma if w.is_cuda else float(sigma)

    @torch.no_grad()
    def step(self, closure: Optional[Any] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, wd = group["lr"], group["weight_decay"]
            iters = group["power_iteration_steps"]
            tasks = []
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise SparseGradientError("SpectralSphereOptimizer does not support sparse gradients")
                st = self.state[p]
                if len(st) == 0:
                    st["momentum_buffer"] = zeros_state_like(p)
                    if p.dim() == 2:
                        st["initial_sigma"] = self._sigma(p, iters)
                decay = 1.0 - lr * wd
                if p.dim() == 2:
                    sigma = self._sigma(p, iters)
                    R = compute_target_radius(p.shape, group["radius_mode"], group["radius_scaler"])
                    r = retraction_scale(sigma, R, group["retract_mode"])
                    st["current_sigma"] = sigma
                    st["target_radius"] = R
                    decay = r * decay
                is2d = p.dim() == 2
                tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(st["momentum_buffer"]),
                                      lr_eff=lr * (muon_lr_scale(p.shape) if is2d else 1.0), decay=decay,
                                      orthogonalize=is2d))
            hp = MuonHyper(mode=MODE_EMA, momentum=group["momentum"], nesterov=group["nesterov"],
                           ns_steps=group["ns_steps"])
            self._engine.step(tasks, hp)
        return loss

    def get_spectral_norms(self) -> dict:
        """``{id(p): {"current_sigma", "target_radius", "initial_sigma"}}`` as Python floats."""
        out = {}
        for group in self.param_groups:
            iters = group.get("power_iteration_steps", 10)
            for p in group["params"]:
                if p.dim() != 2:
                    continue
                st = self.state[p]
                info = {}
                for k in ("current_sigma", "target_radius", "initial_sigma"):
                    if k in st:
                        v = st[k]
                        info[k] = float(v.item()) if isinstance(v, torch.Tensor) else float(v)
                if "initial_sigma" not in st:
                    v = self._sigma(p, iters)
                    info["current_sigma"] = float(v.item()) if isinstance(v, torch.Tensor) else float(v)
                if info:
                    out[id(p)] = info
        return out

    def load_state_dict(self, state_dict: dict) -> None:
        load_index_state_dict(self, state_dict)
