"""TransformerEncoder + FSDP2 + hybrid Muon/AdamW regression workload (counterpart of the
reference's examples/fsdp_distributed.py): 6 post-LN layers, d_model 512, 8 heads, FFN 2048,
batch 32 x seq 512, inputs ~N(0,1), MSE to N(0,1) targets; Muon on 2-D weights, AdamW (lr 1e-3)
on biases / LayerNorm.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/fsdp_distributed.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import argparse
import os
import time

import torch
import torch.distributed as dist

from my_muon_fsdp2_b200 import HybridMuonAdamW
from my_muon_fsdp2_b200.models.encoder import SimpleTransformer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=512)
    a = ap.parse_args()
    cuda = torch.cuda.is_available()
    dist.init_process_group("nccl" if cuda else "gloo")
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dev = "cuda" if cuda else "cpu"
    torch.manual_seed(0)
    model = SimpleTransformer(d_model=512, nhead=8, num_layers=6, dim_feedforward=2048, input_dim=512,
                              output_dim=512).to(dev, torch.bfloat16 if cuda else torch.float32)
    model.apply_fsdp2()
    opt = HybridMuonAdamW(model.parameters(), muon_lr=0.02, adamw_lr=1e-3)
    for step in range(a.steps):
        x = torch.randn(a.batch, a.seq, 512, device=dev, dtype=next(model.parameters()).dtype)
        y = torch.randn_like(x)
        t0 = time.time()
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.mse_loss(model(x).float(), y.float())
        loss.backward()
        opt.step()
        if dist.get_rank() == 0:
            print(f"step {step} loss {loss.item():.4f} {1e3 * (time.time() - t0):.1f} ms")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
