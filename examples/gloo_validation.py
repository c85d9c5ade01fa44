"""CPU / gloo validation of FSDP2 + FSDPMuonOptimizer (the CPU/gloo MLP workload: MLP
512->2048->512, fully_shard per Linear + root, batch 64, MSE on N(0,1) data, seed 0, lr .02,
momentum .95, wd .01, Nesterov, 5 NS steps, 100 steps).  Prints the loss curve and the median
optimizer.step() time.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/gloo_validation.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import statistics
import time

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.device_mesh import init_device_mesh
from torch.distributed.fsdp import fully_shard

from my_muon_fsdp2_b200 import FSDPMuonOptimizer


def main():
    dist.init_process_group("gloo")
    world = dist.get_world_size()
    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(512, 2048), nn.GELU(), nn.Linear(2048, 512))
    for m in model:
        if isinstance(m, nn.Linear):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    opt = FSDPMuonOptimizer(model, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True, ns_steps=5)
    torch.manual_seed(0)
    x, y = torch.randn(64, 512), torch.randn(64, 512)
    times, losses = [], []
    for step in range(100):
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        t0 = time.perf_counter()
        opt.step()
        times.append(time.perf_counter() - t0)
        losses.append(loss.item())
    if dist.get_rank() == 0:
        print(f"loss[0,1,10,99] = {losses[0]:.5f} {losses[1]:.5f} {losses[10]:.5f} {losses[99]:.5f}")
        print(f"median optimizer.step() = {1e3 * statistics.median(times):.1f} ms")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
