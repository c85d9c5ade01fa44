"""Independent restatements of the reference's optimizer math, used as test oracles."""
import torch

from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference


def muon_reference_step(params, grads, bufs, lr, momentum, wd, nesterov, ns_steps):
    """src/muon_fsdp/optimizer.py:102-172 in float64."""
    for p, g, buf in zip(params, grads, bufs):
        buf.lerp_(g, 1 - momentum)
        u = g + momentum * buf if nesterov else buf.clone()
        if p.dim() == 2:
            u = newton_schulz_reference(u, steps=ns_steps)
            m, n = p.shape
            u = u * max(1.0, min(m, n) / max(m, n)) ** 0.5
        if wd != 0:
            p.mul_(1 - lr * wd)
        p.add_(u, alpha=-lr)
