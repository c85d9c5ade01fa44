"""Hybrid Muon (2-D) + AdamW (1-D) training (counterpart of the reference's examples/mixed_adamw.py).

    python examples/mixed_adamw.py --steps 10
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import argparse

import torch

from my_muon_fsdp2_b200 import create_hybrid_optimizer, is_hidden_matrix
from my_muon_fsdp2_b200.models.gpt2 import GPTConfig, GPTModel


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--hidden-only", action="store_true", help="keep embeddings on AdamW")
    a = ap.parse_args()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cfg = GPTConfig(n_layer=4, n_embd=256, n_head=4, vocab_size=4096, n_positions=256)
    model = GPTModel(cfg).to(dev, torch.bfloat16 if dev == "cuda" else torch.float32)
    opt = create_hybrid_optimizer(model, muon_lr=0.02, adamw_lr=1e-3, muon_filter=is_hidden_matrix if a.hidden_only else None)
    print(opt.statistics())
    for step in range(a.steps):
        tok = torch.randint(0, cfg.vocab_size, (8, 129), device=dev)
        opt.zero_grad()
        loss = model(tok[:, :-1], tok[:, 1:])
        loss.backward()
        opt.step()
        print(f"step {step} loss {loss.item():.4f}")


if __name__ == "__main__":
    main()
