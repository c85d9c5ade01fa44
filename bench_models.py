"""Throughput of the two smaller FSDP2 + Muon workloads, this library vs the reference.

  --model encoder : nn.TransformerEncoder, 6 post-LN layers, d_model 512, 8 heads, FFN 2048,
                    dropout 0, bf16; batch 32 x seq 512 per GPU, inputs and MSE targets ~N(0,1);
                    fully_shard per layer + root; Muon on the 2-D weights (lr .02, mom .95,
                    wd .01), AdamW on biases / LayerNorm (lr 1e-3).
  --model gpt2    : GPT-2 small (12 layers, d768, 12 heads, GELU MLP 3072, vocab 50257, ctx 1024,
                    tied embedding), bf16; 16 sequences of 1024 uniform random tokens per GPU,
                    next-token CE; Muon on the hidden 2-D matrices, AdamW on embeddings / LN / bias.

--impl ours      : this library's models and kernels (GPT-2) or torch's own module (encoder), with
                   MuonOptimizer + FusedAdamW.
--impl reference : the reference's ``muon_fsdp.MuonOptimizer`` (from baseline/_ref, unmodified) +
                   ``torch.optim.AdamW`` on the same workload (GPT-2 from transformers).

Timing: W warm-up steps, then K steps between CUDA events on the launching stream, max over
ranks; one JSON line from rank 0.  ``value`` is tokens/s over all GPUs.

    python bench_models.py --model gpt2 [--steps K --warmup W --impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_models.py --model encoder
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["encoder", "gpt2"], default="gpt2")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--fsdp", choices=["fsdp2", "symm"], default="fsdp2",
                    help="gpt2 (ours): fully_shard everywhere, or the block linears on the fused collectives")
    return ap.parse_args()


def init():
    if "RANK" not in os.environ:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def ref_muon():
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "muon_fsdp")):
        raise RuntimeError("reference package not installed under baseline/_ref")
    sys.path.insert(0, ref)
    from muon_fsdp import MuonOptimizer

    return MuonOptimizer


def build_encoder(impl, dev, fsdp="fsdp2"):
    from torch.distributed.fsdp import fully_shard

    torch.manual_seed(0)
    layer = torch.nn.TransformerEncoderLayer(512, 8, 2048, 0.0, batch_first=True)
    model = torch.nn.Sequential(torch.nn.TransformerEncoder(layer, 6, enable_nested_tensor=False))
    model = model.to(dev, torch.bfloat16)
    for lyr in model[0].layers:
        fully_shard(lyr)
    fully_shard(model)
    mats = [p for p in model.parameters() if p.dim() == 2]
    rest = [p for p in model.parameters() if p.dim() != 2]
    B, T = 32, 512

    def batch(step):
        g = torch.Generator(device="cpu").manual_seed(step)
        x = torch.randn(B, T, 512, generator=g).to(dev, torch.bfloat16)
        y = torch.randn(B, T, 512, generator=g).to(dev, torch.bfloat16)
        return x, y

    def loss_fn(x, y):
        return torch.nn.functional.mse_loss(model(x).float(), y.float())

    return model, mats, rest, batch, loss_fn, B * T


def build_gpt2(impl, dev, fsdp="fsdp2"):
    from torch.distributed.fsdp import fully_shard

    torch.manual_seed(0)
    B, T, V = 16, 1024, 50257
    if impl == "ours":
        from my_muon_fsdp2_b200.models.gpt2 import GPT2SmallConfig, GPTModel

        model = GPTModel(GPT2SmallConfig()).to(dev, torch.bfloat16)
        if fsdp == "symm":
            from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

            apply_symm_fsdp(model, blocks_attr="h")
        else:
            model.configure_fsdp()
        names = set(model.muon_param_names())

        def loss_fn(x, y):
            return model(x, y)
    else:
        from transformers import GPT2Config, GPT2LMHeadModel

        cfg = GPT2Config(vocab_size=V, n_positions=T, n_embd=768, n_layer=12, n_head=12, resid_pdrop=0.0,
                         embd_pdrop=0.0, attn_pdrop=0.0, attn_implementation="sdpa", use_cache=False)
        model = GPT2LMHeadModel(cfg).to(dev, torch.bfloat16)
        for blk in model.transformer.h:
            fully_shard(blk)
        fully_shard(model)
        names = {n for n, p in model.named_parameters() if p.dim() == 2 and ".h." in n}

        def loss_fn(x, y):
            return model(input_ids=x, labels=x).loss
    mats = [p for n, p in model.named_parameters() if n in names]
    rest = [p for n, p in model.named_parameters() if n not in names]

    def batch(step):
        g = torch.Generator(device="cpu").manual_seed(step)
        t = torch.randint(0, V, (B, T + 1), generator=g).to(dev)
        return t[:, :-1].contiguous(), t[:, 1:].contiguous()

    return model, mats, rest, batch, loss_fn, B * T


def main():
    args = parse()
    rank, world, local = init()
    dev = torch.device("cuda", local)
    try:
        build = build_encoder if args.model == "encoder" else build_gpt2
        model, mats, rest, batch, loss_fn, tokens_per_gpu = build(args.impl, dev, args.fsdp)
        if args.impl == "ours":
            from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer

            opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95, weight_decay=0.01),
                    FusedAdamW(rest, lr=1e-3, weight_decay=0.01)]
            ctl = getattr(model, "_symm_fsdp", None)
            for o in opts if ctl is not None else []:
                ctl.attach_optimizer(o)
        else:
            Muon = ref_muon()
            opts = [Muon(mats, lr=0.02, momentum=0.95, weight_decay=0.01),
                    torch.optim.AdamW(rest, lr=1e-3, weight_decay=0.01)]
    except Exception as e:
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "model": args.model,
                                  "unavailable": f"{type(e).__name__}: {e}"[:300]}))
            dist.destroy_process_group()
            return
        raise
    data = [batch(s) for s in range(2)]

    def step(s):
        x, y = data[s % 2]
        loss = loss_fn(x, y)
        loss.backward()
        for o in opts:
            o.step()
        for o in opts:
            o.zero_grad(set_to_none=True)
        return loss.detach()

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(args.steps):
        loss = step(s)
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / args.steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({"metric": f"{args.model} FSDP2+Muon tokens/s", "impl": args.impl, "value":
                          world * tokens_per_gpu / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
                          "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                          "data": "synthetic; random-init weights", "final_loss": float(loss.item()),
                          "config": {"model": args.model, "tokens_per_gpu": tokens_per_gpu,
                                     "parallelism": f"fsdp{world}", "fsdp_impl": args.fsdp}}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
