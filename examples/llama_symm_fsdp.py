"""Llama-style model with the fused FSDP collectives: the block linears live on symmetric
memory (all-gather fused into the first forward GEMM of each step, reduce-scatter on a side
stream), the rest of the model on FSDP2; Muon on the attention/FFN matrices, AdamW on the rest;
gradient accumulation with a synchronising last micro-batch, gradient clipping, per-step metrics.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/llama_symm_fsdp.py      # B200s
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/llama_symm_fsdp.py      # CPU/gloo too
    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 examples/llama_symm_fsdp.py --replicas 2   # HSDP

On CPU (gloo) the same module runs its collectives through torch.distributed.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import argparse

import torch
import torch.distributed as dist

from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer
from my_muon_fsdp2_b200.models.llama import Llama, LlamaConfig
from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp
from my_muon_fsdp2_b200.parallel.fault import init_distributed
from my_muon_fsdp2_b200.train import Trainer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--grad-accum", type=int, default=2)
    ap.add_argument("--replicas", type=int, default=1,
                    help="HSDP: a (replicas, world / replicas) mesh; the linears are sharded over the second dim")
    a = ap.parse_args()
    cuda = torch.cuda.is_available()
    # NCCL on GPUs (gloo on CPU) with a collective timeout and async error handling
    job = init_distributed(timeout_s=300.0)
    if not dist.is_initialized():
        sys.exit("llama_symm_fsdp.py shards the model over a process group: launch it with torchrun "
                 "(e.g. torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/llama_symm_fsdp.py)")
    rank, dev = job["rank"], job["device"]
    torch.manual_seed(0)
    cfg = LlamaConfig.tiny(dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024, vocab_size=2048, n_layers=2)
    model = Llama(cfg).to(dev, torch.bfloat16 if cuda else torch.float32)
    mesh = None
    if a.replicas > 1:
        from torch.distributed.device_mesh import init_device_mesh

        world = dist.get_world_size()
        mesh = init_device_mesh(dev.type, (a.replicas, world // a.replicas), mesh_dim_names=("replicate", "shard"))
    ctl = apply_symm_fsdp(model, mesh=mesh)
    names = set(model.muon_param_names())
    opts = [MuonOptimizer([p for n, p in model.named_parameters() if n in names], lr=0.02, weight_decay=0.01),
            FusedAdamW([p for n, p in model.named_parameters() if n not in names], lr=1e-3)]
    trainer = Trainer(model, opts, grad_accum=a.grad_accum, device=dev, max_grad_norm=1.0)
    for step in range(a.steps):
        g = torch.Generator().manual_seed(1000 * step + rank)
        batch = torch.randint(0, cfg.vocab_size, (a.grad_accum, 1, a.seq + 1), generator=g)
        loss = trainer.train_step(batch)
        m = trainer.last_metrics
        if rank == 0:
            print(f"step {step} loss {loss:.4f} grad_norm {float(m['grad_norm']):.3f} "
                  f"resident_weights {m.get('symm_fsdp/resident_weights')} rs_mode {ctl.rs_mode}")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
