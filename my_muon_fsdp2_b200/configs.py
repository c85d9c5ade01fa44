"""The five benchmark workloads of this library, as data (the reference has no config system:
its settings live in example argparse blocks, e.g. examples/train_gpt.py:470-493).

Each entry names the model, the per-GPU batch, the optimizers and the command that measures it;
``python -m my_muon_fsdp2_b200.cli configs`` prints them.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Dict


@dataclass(frozen=True)
class BenchConfig:
    name: str
    model: str
    gpus: str
    dtype: str
    batch_per_gpu: str
    optimizer: str
    command: str


WORKLOADS: Dict[str, BenchConfig] = {
    "mlp_gloo": BenchConfig(
        name="mlp_gloo", model="MLP Linear(512->2048)-GELU-Linear(2048->512), fully_shard per Linear + root",
        gpus="CPU gloo, world size 2", dtype="fp32", batch_per_gpu="64 x 512, MSE to N(0,1) targets, seed 0",
        optimizer="FSDPMuonOptimizer lr .02 momentum .95 wd .01 nesterov ns 5; 100 steps",
        command="torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/gloo_validation.py"),
    "encoder": BenchConfig(
        name="encoder", model="nn.TransformerEncoder 6 post-LN layers, d512, 8 heads, FFN 2048, dropout 0",
        gpus="1-8 B200", dtype="bf16", batch_per_gpu="32 x 512 tokens, inputs and MSE targets N(0,1)",
        optimizer="Muon on 2-D weights (lr .02) + AdamW on bias / LayerNorm (lr 1e-3)",
        command="torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_models.py --model encoder"),
    "gpt2_small": BenchConfig(
        name="gpt2_small", model="GPT-2 small 124M (12 layers, d768, 12 heads, GELU 3072, vocab 50257, ctx 1024, tied)",
        gpus="1-8 B200", dtype="bf16", batch_per_gpu="16 x 1024 uniform random tokens, next-token CE",
        optimizer="Muon on hidden 2-D matrices (lr .02, momentum .95, wd .01) + AdamW on the rest",
        command="torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_models.py --model gpt2"),
    "llama3_8b": BenchConfig(
        name="llama3_8b", model="Llama-3 8B (32 layers, d4096, 32q/8kv heads, hd128, SwiGLU 14336, RMSNorm, "
        "RoPE 500000, vocab 128256)", gpus="1/2/4/8 B200", dtype="bf16 params, fp32 momentum",
        batch_per_gpu="1 x 4096 tokens, grad accumulation 4",
        optimizer="Muon on attention/FFN matrices (lr .02, mom .95, wd .01) + AdamW on the rest",
        command="torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N"),
    "muon_sweep": BenchConfig(
        name="muon_sweep", model="row-sharded bf16 N(0,1) momentum: 4096x4096, 1024x4096, 4096x14336, "
        "14336x4096, 8192x28672", gpus="2/4/8 B200", dtype="bf16",
        batch_per_gpu="one shard of each matrix", optimizer="gather + 5 quintic NS iterations + scatter-update",
        command="torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_ns.py"),
}


def describe() -> Dict[str, dict]:
    return {k: asdict(v) for k, v in WORKLOADS.items()}
