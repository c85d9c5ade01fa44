"""Spectral-Sphere vs Muon on a small MLP, tracking the top singular value (counterpart of the
reference's examples/train_sso.py)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import torch
import torch.nn as nn

from my_muon_fsdp2_b200 import MuonOptimizer, SpectralSphereOptimizer


def run(opt_cls, **kw):
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(128, 256), nn.GELU(), nn.Linear(256, 64))
    opt = opt_cls(model.parameters(), **kw)
    x, y = torch.randn(256, 128), torch.randn(256, 64)
    for _ in range(50):
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        opt.step()
    sig = [torch.linalg.matrix_norm(m.weight.detach(), 2).item() for m in model if isinstance(m, nn.Linear)]
    return loss.item(), sig


if __name__ == "__main__":
    print("muon", run(MuonOptimizer, lr=0.02))
    print("sso ", run(SpectralSphereOptimizer, lr=0.02, radius_mode="spectral_mup"))
