"""Worker for the multi-GPU tests (launched with torchrun by tests/test_gpu_distributed.py).

Trains a small FSDP2 Llama for a few steps with MuonOptimizer (+ FusedAdamW) using the given
exchange (``nccl`` all-to-all or ``p2p`` symmetric memory) and saves the full parameters."""
import argparse
import datetime
import os

import torch
import torch.distributed as dist


def build(world, local, comm, sharded=True):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer
    from my_muon_fsdp2_b200.models.llama import Llama, LlamaConfig, apply_fsdp

    torch.manual_seed(0)
    cfg = LlamaConfig.tiny(dim=256, n_heads=4, n_kv_heads=2, ffn_dim=640, vocab_size=1024, n_layers=2)
    model = Llama(cfg).to(dtype=torch.bfloat16)
    model = model.to(f"cuda:{local}")
    if sharded:
        apply_fsdp(model, init_device_mesh("cuda", (world,)))
    names = set(model.muon_param_names())
    opts = [MuonOptimizer([p for n, p in model.named_parameters() if n in names], lr=0.02, weight_decay=0.01,
                          comm=comm),
            FusedAdamW([p for n, p in model.named_parameters() if n not in names], lr=1e-3)]
    return model, opts, cfg


def train(model, opts, cfg, steps, device):
    losses = []
    for s in range(steps):
        g = torch.Generator().manual_seed(s)
        tok = torch.randint(0, cfg.vocab_size, (2, 65), generator=g).to(device)
        loss = model(tok[:, :-1], tok[:, 1:])
        loss.backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
        losses.append(loss.item())
    return losses


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="nccl")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    model, opts, cfg = build(world, local, a.comm)
    losses = train(model, opts, cfg, a.steps, f"cuda:{local}")
    full = {n: p.full_tensor().float().cpu() for n, p in model.named_parameters()}
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(local)
    if rank == 0:
        torch.save({"losses": losses, "params": full}, a.out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
