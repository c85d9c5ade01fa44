"""Multi-tensor fused AdamW (decoupled weight decay, fp32 moments).

Used for the non-Muon parameters (embeddings, norms, biases, LM head) of the hybrid setups.
CUDA parameters: one ``adamw_multi`` kernel launch per (param dtype, grad dtype) bucket.
CPU parameters: the same math with PyTorch ops.  State keys ``exp_avg``, ``exp_avg_sq``, ``step``
follow torch.optim.AdamW / the reference's hybrid AdamW branch (examples/mixed_adamw.py:310-355).
"""
from __future__ import annotations

import math
from collections import OrderedDict

import torch
from torch.optim import Optimizer

from ._common import load_index_state_dict, local_of, zeros_state_like
from .errors import InvalidParameterError, SparseGradientError


def adamw_update_(params, grads, exp_avgs, exp_avg_sqs, step: int, lr: float, beta1: float, beta2: float,
                  eps: float, weight_decay: float) -> None:
    """Apply one AdamW step (bias-corrected for ``step`` >= 1) to lists of local tensors."""
    if not params:
        return
    bc1 = 1.0 - beta1 ** step
    bc2s = math.sqrt(1.0 - beta2 ** step)
    if params[0].is_cuda:
        from .._ext import ext

        E = ext()
        buckets: "OrderedDict" = OrderedDict()
        for i, (p, g) in enumerate(zip(params, grads)):
            buckets.setdefault((p.dtype, g.dtype), []).append(i)
        for _, idx in buckets.items():
            E.adamw([params[i] for i in idx], [grads[i].contiguous() for i in idx], [exp_avgs[i] for i in idx],
                    [exp_avg_sqs[i] for i in idx], lr, beta1, beta2, eps, weight_decay, bc1, bc2s)
        return
    for p, g, m, v in zip(params, grads, exp_avgs, exp_avg_sqs):
        gf = g.to(m.dtype)
        m.lerp_(gf, 1 - beta1)
        v.mul_(beta2).addcmul_(gf, gf, value=1 - beta2)
        if weight_decay != 0:
            p.mul_(1 - lr * weight_decay)
        denom = (v.sqrt() / bc2s).add_(eps)
        p.add_((m / denom).to(p.dtype), alpha=-lr / bc1)


class FusedAdamW(Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.01):
        if lr < 0:
            raise InvalidParameterError(f"Invalid learning rate: {lr}")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise InvalidParameterError(f"Invalid betas: {betas}")
        if eps < 0:
            raise InvalidParameterError(f"Invalid epsilon value: {eps}")
        if weight_decay < 0:
            raise InvalidParameterError(f"Invalid weight_decay value: {weight_decay}")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            by_step: "OrderedDict[int, list]" = OrderedDict()
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise SparseGradientError("FusedAdamW does not support sparse gradients")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = zeros_state_like(p, fp32_on_cuda=True)
                    st["exp_avg_sq"] = zeros_state_like(p, fp32_on_cuda=True)
                st["step"] += 1
                by_step.setdefault(st["step"], []).append(p)
            for step, ps in by_step.items():
                adamw_update_([local_of(p) for p in ps], [local_of(p.grad) for p in ps],
                              [local_of(self.state[p]["exp_avg"]) for p in ps],
                              [local_of(self.state[p]["exp_avg_sq"]) for p in ps], step, group["lr"], b1, b2,
                              group["eps"], group["weight_decay"])
        return loss

    def load_state_dict(self, state_dict: dict) -> None:
        load_index_state_dict(self, state_dict)
