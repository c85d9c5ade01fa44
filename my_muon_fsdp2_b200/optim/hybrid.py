"""Hybrid Muon (2-D matrices) + AdamW (everything else) optimizer.

Parity with the reference example builder (``examples/mixed_adamw.py:191-485``):
``HybridMuonAdamW`` (single optimizer routing by parameter dimension),
``HybridMuonAdamWOptimizer`` (model wrapper with ``statistics()`` and delegates) and
``create_hybrid_optimizer``.  Muon branch: EMA momentum, no Nesterov, NS, unit dimension scale,
decoupled weight decay with ``muon_lr``.  AdamW branch: betas/eps/decoupled weight decay with
``adamw_lr``; hyper-parameters are read from the ``muon_*`` / ``adamw_*`` group keys as in the
reference (mixed_adamw.py:277-281, 317-321).

Differences: the AdamW bias correction uses the incremented step (the reference divides by
zero on its first step, mixed_adamw.py:332-343; ``reference_compat=True`` reproduces that
failure), and a group may set ``use_muon`` to override the dimension rule (e.g. keep embeddings
on AdamW).  Both branches run as fused multi-tensor kernels on CUDA.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Callable, Dict, List, Optional

import torch
import torch.nn as nn
from torch import optim

from ..ops.newton_schulz import muon_lr_scale
from ..parallel.muon_engine import MODE_EMA, MuonHyper, MuonTask
from ._common import default_engine, load_index_state_dict, local_of, zeros_state_like
from .adamw import adamw_update_
from .errors import SparseGradientError


class HybridMuonAdamW(optim.Optimizer):
    def __init__(self, params, muon_lr: float = 0.02, adamw_lr: float = 1e-3, muon_momentum: float = 0.95,
                 adamw_beta1: float = 0.9, adamw_beta2: float = 0.999, adamw_eps: float = 1e-8,
                 muon_weight_decay: float = 0.0, adamw_weight_decay: float = 0.01, ns_steps: int = 5, *,
                 muon_nesterov: bool = False, reference_compat: bool = False, process_group=None,
                 comm: str = "auto"):
        defaults = dict(muon_lr=muon_lr, adamw_lr=adamw_lr, muon_momentum=muon_momentum, adamw_beta1=adamw_beta1,
                        adamw_beta2=adamw_beta2, adamw_eps=adamw_eps, muon_weight_decay=muon_weight_decay,
                        adamw_weight_decay=adamw_weight_decay, ns_steps=ns_steps, muon_nesterov=muon_nesterov)
        super().__init__(params, defaults)
        self.reference_compat = reference_compat
        self._engine = default_engine(process_group, comm)

    def _is_muon(self, group, p) -> bool:
        use = group.get("use_muon")
        return bool(use) if use is not None else p.dim() == 2

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            muon, adam = [], []
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise SparseGradientError("HybridMuonAdamW does not support sparse gradients")
                (muon if self._is_muon(group, p) else adam).append(p)
            if muon:
                self._muon_step(group, muon)
            if adam:
                self._adamw_step(group, adam)
        return loss

    def _muon_step(self, group, ps: List[torch.Tensor]) -> None:
        lr, wd = group["muon_lr"], group["muon_weight_decay"]
        tasks = []
        for p in ps:
            st = self.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = zeros_state_like(p)
            is2d = p.dim() == 2
            tasks.append(MuonTask(param=p, grad=p.grad, buf=local_of(st["momentum_buffer"]),
                                  lr_eff=lr * (muon_lr_scale(p.shape) if is2d else 1.0), decay=1.0 - lr * wd,
                                  orthogonalize=is2d))
        self._engine.step(tasks, MuonHyper(mode=MODE_EMA, momentum=group["muon_momentum"],
                                           nesterov=group.get("muon_nesterov", False), ns_steps=group["ns_steps"]))

    def _adamw_step(self, group, ps: List[torch.Tensor]) -> None:
        by_step: "OrderedDict[int, list]" = OrderedDict()
        for p in ps:
            st = self.state[p]
            if len(st) == 0:
                st["exp_avg"] = zeros_state_like(p)
                st["exp_avg_sq"] = zeros_state_like(p)
                st["step"] = 0
            step = st["step"]
            st["step"] = step + 1
            if self.reference_compat:
                if step == 0:
                    raise ZeroDivisionError(
                        "reference_compat: the reference hybrid AdamW computes its bias correction from the "
                        "pre-increment step and divides by zero on the first step (mixed_adamw.py:332-343)")
                by_step.setdefault(step, []).append(p)
            else:
                by_step.setdefault(step + 1, []).append(p)
        for step, lst in by_step.items():
            adamw_update_([local_of(p) for p in lst], [local_of(p.grad) for p in lst],
                          [local_of(self.state[p]["exp_avg"]) for p in lst],
                          [local_of(self.state[p]["exp_avg_sq"]) for p in lst], step, group["adamw_lr"],
                          group["adamw_beta1"], group["adamw_beta2"], group["adamw_eps"], group["adamw_weight_decay"])

    def load_state_dict(self, state_dict: dict) -> None:
        load_index_state_dict(self, state_dict)


def is_hidden_matrix(name: str, p: torch.Tensor) -> bool:
    """2-D weights except embeddings / LM head (Muon on hidden matrices, AdamW on the rest)."""
    if p.dim() != 2:
        return False
    low = name.lower()
    return not any(k in low for k in ("embed", "wte", "wpe", "lm_head", "tok_emb", "pos_emb", "output.weight"))


class HybridMuonAdamWOptimizer:
    """Wrapper that splits a model's parameters into a Muon group and an AdamW group."""

    def __init__(self, model: nn.Module, muon_lr: float = 0.02, adamw_lr: float = 1e-3, muon_momentum: float = 0.95,
                 adamw_beta1: float = 0.9, adamw_beta2: float = 0.999, adamw_eps: float = 1e-8,
                 muon_weight_decay: float = 0.0, adamw_weight_decay: float = 0.01, ns_steps: int = 5,
                 fsdp_model: Optional[nn.Module] = None, *,
                 muon_filter: Optional[Callable[[str, torch.Tensor], bool]] = None, **kwargs):
        self.model = model
        self.fsdp_model = fsdp_model
        self._classify_parameters(model, muon_filter)
        self.optimizer = HybridMuonAdamW(
            params=[{"params": self.muon_params, "use_muon": True},
                    {"params": self.adamw_params, "use_muon": False}],
            muon_lr=muon_lr, adamw_lr=adamw_lr, muon_momentum=muon_momentum, adamw_beta1=adamw_beta1,
            adamw_beta2=adamw_beta2, adamw_eps=adamw_eps, muon_weight_decay=muon_weight_decay,
            adamw_weight_decay=adamw_weight_decay, ns_steps=ns_steps, **kwargs)

    def _classify_parameters(self, model: nn.Module, muon_filter=None) -> None:
        self.muon_params: List[nn.Parameter] = []
        self.adamw_params: List[nn.Parameter] = []
        for name, p in model.named_parameters():
            if not p.requires_grad:
                continue
            use = muon_filter(name, p) if muon_filter is not None else p.dim() == 2
            (self.muon_params if use else self.adamw_params).append(p)

    @property
    def param_groups(self):
        return self.optimizer.param_groups

    def statistics(self) -> Dict[str, float]:
        mc = sum(p.numel() for p in self.muon_params)
        ac = sum(p.numel() for p in self.adamw_params)
        tot = mc + ac
        return {"muon_params": len(self.muon_params), "muon_parameters": mc, "adamw_params": len(self.adamw_params),
                "adamw_parameters": ac, "total_params": tot, "muon_ratio": mc / tot * 100 if tot else 0}

    def step(self, closure=None):
        return self.optimizer.step(closure)

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.optimizer.zero_grad(set_to_none)

    def state_dict(self) -> Dict:
        return self.optimizer.state_dict()

    def load_state_dict(self, state_dict: Dict) -> None:
        self.optimizer.load_state_dict(state_dict)


def create_hybrid_optimizer(model: nn.Module, muon_lr: float = 0.02, adamw_lr: float = 1e-3,
                            muon_weight_decay: float = 0.0, adamw_weight_decay: float = 0.01, use_fsdp: bool = False,
                            fsdp_model: Optional[nn.Module] = None, **kwargs) -> HybridMuonAdamWOptimizer:
    """Builder with the reference's signature (mixed_adamw.py:455-485)."""
    return HybridMuonAdamWOptimizer(model=model, muon_lr=muon_lr, adamw_lr=adamw_lr,
                                    muon_weight_decay=muon_weight_decay, adamw_weight_decay=adamw_weight_decay,
                                    fsdp_model=fsdp_model if use_fsdp else None, **kwargs)
