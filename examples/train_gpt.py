"""GPT-2 training with Muon on FSDP2 (counterpart of the reference's examples/train_gpt.py).

    python examples/train_gpt.py --model small --steps 20                      # 1 GPU
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/train_gpt.py --fsdp
Muon (lr .02, momentum .95, wd .01) on the hidden 2-D matrices, AdamW on embeddings/LN/bias.
Saves ``<save_dir>/muon_gpt2_<model>.pt`` (model_state_dict, optimizer_state_dict, epoch, loss)
and resumes from it with ``--resume``.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # repo checkout

import argparse
import os
import time

import torch
import torch.distributed as dist

from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer
from my_muon_fsdp2_b200.models.gpt2 import GPT2LargeConfig, GPT2MediumConfig, GPT2SmallConfig, GPTModel
from my_muon_fsdp2_b200.train import Trainer, load_checkpoint, save_checkpoint


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["small", "medium", "large"], default="small")
    ap.add_argument("--batch", type=int, default=16, help="sequences per GPU per step")
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--grad-accum", type=int, default=1)
    ap.add_argument("--fsdp", action="store_true")
    ap.add_argument("--save-dir", default="checkpoints")
    ap.add_argument("--resume", action="store_true")
    a = ap.parse_args()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if a.fsdp:
        dist.init_process_group("nccl" if dev == "cuda" else "gloo")
        if dev == "cuda":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    cfg = {"small": GPT2SmallConfig, "medium": GPT2MediumConfig, "large": GPT2LargeConfig}[a.model]()
    model = GPTModel(cfg).to(dev, torch.bfloat16 if dev == "cuda" else torch.float32)
    if a.fsdp:
        model.configure_fsdp()
    muon_names = set(model.muon_param_names())
    opts = [MuonOptimizer([p for n, p in model.named_parameters() if n in muon_names], lr=0.02, momentum=0.95,
                          weight_decay=0.01),
            FusedAdamW([p for n, p in model.named_parameters() if n not in muon_names], lr=1e-3, weight_decay=0.01)]
    name = f"gpt2_{a.model}"
    if a.resume and os.path.exists(os.path.join(a.save_dir, f"muon_{name}.pt")):
        info = load_checkpoint(os.path.join(a.save_dir, f"muon_{name}.pt"), model, opts)
        print(f"resumed from epoch {info['epoch']} (loss {info['loss']})")
    trainer = Trainer(model, opts, grad_accum=a.grad_accum)
    loss = float("nan")
    for step in range(a.steps):
        batch = torch.randint(1, cfg.vocab_size, (a.grad_accum, a.batch, a.seq + 1)).pin_memory() \
            if dev == "cuda" else torch.randint(1, cfg.vocab_size, (a.grad_accum, a.batch, a.seq + 1))
        t0 = time.time()
        loss = trainer.train_step(batch)
        if not a.fsdp or dist.get_rank() == 0:
            print(f"step {step} loss {loss:.4f} {1e3 * (time.time() - t0):.1f} ms")
    save_checkpoint(a.save_dir, name, model, opts, epoch=a.steps, loss=loss)
    if a.fsdp:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
