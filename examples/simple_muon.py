"""Minimal single-process Muon example on an MLP (counterpart of the reference's simple_muon.py)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import torch
import torch.nn as nn

from my_muon_fsdp2_b200 import MuonOptimizer


def main():
    torch.manual_seed(0)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model = nn.Sequential(nn.Linear(512, 2048), nn.GELU(), nn.Linear(2048, 512)).to(dev)
    opt = MuonOptimizer(model.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True)
    x, y = torch.randn(64, 512, device=dev), torch.randn(64, 512, device=dev)
    for step in range(20):
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        opt.step()
        print(f"step {step} loss {loss.item():.5f}")


if __name__ == "__main__":
    main()
