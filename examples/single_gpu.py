"""One process, no process group: the ``fsdp2_utils`` API outside a distributed job
(counterpart of the reference's examples_new/single_gpu.py).

The model-first ``fsdp2_utils.MuonOptimizer`` trains a 256 -> 512 -> 256 GELU MLP for three steps
on MSE, ``zeropower_via_newtonschulz5`` orthogonalises a 256 x 512 matrix, and the comm / DTensor
helpers report the single-process fallbacks.  On a CUDA machine the model runs on ``cuda:0``
(the Newton-Schulz chain then runs on the tcgen05 kernels); otherwise on the CPU.

    python examples/single_gpu.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import torch
import torch.nn as nn
import torch.nn.functional as F

from my_muon_fsdp2_b200.fsdp2_utils import (
    MuonOptimizer,
    get_world_size,
    is_distributed,
    is_dtensor,
    zeropower_via_newtonschulz5,
)


def main() -> int:
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    print(f"distributed: {is_distributed()}  world size: {get_world_size()}  device: {dev}")

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 256)).to(dev)
    print(f"parameters: {sum(p.numel() for p in model.parameters()):,}")
    for name, p in model.named_parameters():
        print(f"  {name}: {tuple(p.shape)}")

    opt = MuonOptimizer(model, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=False, ns_steps=5)
    x, y = torch.randn(32, 256, device=dev), torch.randn(32, 256, device=dev)
    losses = []
    for step in range(3):
        opt.zero_grad()
        loss = F.mse_loss(model(x), y)
        loss.backward()
        opt.step()
        losses.append(loss.item())
        print(f"step {step + 1}: loss {losses[-1]:.6f}")

    # Newton-Schulz on a 256 x 512 Gaussian (well conditioned: sigma_min / sigma_max ~ 0.17).
    # The quintic's fixed point is an orthogonal-like factor with singular values in roughly
    # [0.7, 1.2], so W W^T is near (not at) the identity.
    g = torch.randn(256, 512, device=dev)
    w = zeropower_via_newtonschulz5(g, steps=5).float()
    sv = torch.linalg.svdvals(w.cpu())
    print(f"Newton-Schulz singular values: min {sv.min():.3f} max {sv.max():.3f}  "
          f"||W W^T - I||_F = {(w @ w.T - torch.eye(256, device=dev)).norm().item():.3f}")

    print(f"plain tensor is_dtensor: {is_dtensor(torch.randn(4, 4))}")
    ok = all(l == l for l in losses) and 0.5 < float(sv.min()) and float(sv.max()) < 1.3
    print("single-process example done" if ok else "single-process example FAILED")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
