"""HSDP (replicate x shard) training with HDSPMuonOptimizer on a real 2-D mesh.

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 examples/hdsp_training.py --dp 2 --fsdp 2
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import argparse
import os

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.fsdp import fully_shard

from my_muon_fsdp2_b200 import HDSPMuonOptimizer, HSDPConfig


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--fsdp", type=int, default=2)
    a = ap.parse_args()
    cuda = torch.cuda.is_available()
    dist.init_process_group("nccl" if cuda else "gloo")
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dev = "cuda" if cuda else "cpu"
    cfg = HSDPConfig(dp_size=a.dp, fsdp_size=a.fsdp)
    mesh = cfg.create_device_mesh()
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(512, 2048), nn.GELU(), nn.Linear(2048, 512)).to(dev)
    for m in model:
        if isinstance(m, nn.Linear):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    opt = HDSPMuonOptimizer(model, device_mesh=mesh, **cfg.to_dict())
    for step in range(10):
        x, y = torch.randn(64, 512, device=dev), torch.randn(64, 512, device=dev)
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        opt.step()
        if dist.get_rank() == 0:
            print(f"step {step} loss {loss.item():.4f}")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
