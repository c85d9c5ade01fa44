"""Headline benchmark: Llama-3-8B FSDP2 + Muon training throughput (tokens/s) on N B200 GPUs.

Workload (one optimizer step per rank): 4 micro-batches (grad accumulation) of 1 sequence x 4096
uniform random tokens, bf16 parameters/compute, fp32 Muon momentum; Muon (lr 0.02, momentum
0.95, weight decay 0.01, 5 NS steps) on every attention/FFN matrix, AdamW (lr 1e-3, wd 0.01) on
embeddings, norms and the LM head.  The block linears are sharded over the ranks on symmetric
memory (``apply_symm_fsdp``; ``--fsdp fsdp2`` for plain ``fully_shard`` on every decoder layer);
the rest of the model is under ``fully_shard`` on several ranks and unsharded on one.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Timing: W untimed steps, then K steps bracketed by barrier + synchronize, timed with CUDA events
on the launching stream; the MAX over ranks is reported.  The per-step working set (16 GB of
weights, tens of GB of activations) is far larger than the 126 MB L2, so no L2 flush is needed.
A second K-step loop measures the same metric end to end through ``Trainer.train_step`` (host
->device copy of the pinned token batch and a device->host read of the loss every step).
Rank 0 prints one JSON line.

``--impl reference`` runs the unmodified reference package (installed under baseline/_ref) on a
stock ``transformers`` Llama with the same config, FSDP2 wrapping, data and hyper-parameters.
Its steps take tens of seconds, so past ``--ref-budget-s`` of wall clock it times fewer steps
(warm-up 3, at least 1 timed and 1 end-to-end step) and reports the counts it ran.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "Llama-8B FSDP2+Muon tokens/s at 1/2/4/8 B200; Muon optimizer.step() ms"
MODEL_DESC = "Llama-3-8B (32 layers, d4096, 32q/8kv heads, hd128, SwiGLU 14336, RMSNorm, RoPE 500000, vocab 128256)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--grad-accum", type=int, default=4)
    ap.add_argument("--micro-bs", type=int, default=1)
    ap.add_argument("--layers", type=int, default=32, help="debug only: fewer layers is not the named config")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ref-budget-s", type=float, default=520.0,
                    help="reference arm: wall-clock budget of the whole run; past it the timed steps are cut "
                         "(to at least 1, warm-up to 3, one end-to-end step) and the JSON line says so")
    ap.add_argument("--rs-mode", choices=["overlap", "fused"], default="overlap",
                    help="symm: reduce-scatter on a side stream (overlap) or from the GEMM epilogue (fused)")
    ap.add_argument("--keep-gathered", action="store_true",
                    help="FSDP2 modules stay gathered between the micro-batches of a step (Trainer keep_gathered)")
    ap.add_argument("--root", choices=["shard", "replicate"], default="replicate",
                    help="--fsdp symm on several GPUs: the embedding, norms and LM head under fully_shard, or "
                         "replicated with one gradient all-reduce per step")
    ap.add_argument("--root-allreduce", choices=["hook", "deferred"], default="hook",
                    help="--root replicate: launch each gradient's all-reduce from its hook, or all at the "
                         "end of the backward and wait before the optimizer steps")
    ap.add_argument("--no-phases", action="store_true",
                    help="do not record the per-phase events (forward / backward per micro-batch, optimizer); "
                         "they are read after the timed loop, so they add no synchronisation to it")
    ap.add_argument("--fsdp", choices=["fsdp2", "symm"], default="symm",
                    help="fsdp2: fully_shard everywhere; symm: block linears on symmetric memory with the "
                         "fused all-gather GEMM / GEMM reduce-scatter kernels, the rest fully_shard")
    return ap.parse_args()


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def init_dist():
    if "RANK" not in os.environ:
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(free_port()))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


# The reference publishes no throughput for this workload, so there is no published number to
# divide by: vs_baseline stays null.
PUBLISHED_TOKENS_PER_S = None


def baseline_value():
    return PUBLISHED_TOKENS_PER_S


def synthetic_tokens(step: int, ga: int, mbs: int, seq: int, vocab: int, rank: int, device="cpu"):
    g = torch.Generator().manual_seed(10007 * step + rank)
    return torch.randint(0, vocab, (ga, mbs, seq + 1), generator=g).to(device)


# ------------------------------------------------------------------------------ our arm
def build_ours(args, world, local):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer
    from my_muon_fsdp2_b200.models.llama import Llama, LlamaConfig, apply_fsdp

    cfg = LlamaConfig.llama3_8b()
    cfg.n_layers = args.layers
    mesh = init_device_mesh("cuda", (world,))
    with torch.device("meta"):
        model = Llama(cfg).to(torch.bfloat16)
    ctl = None
    if args.fsdp == "symm":
        from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

        ctl = apply_symm_fsdp(model, mesh, device=torch.device("cuda", local), rs_mode=args.rs_mode, root=args.root,
                              root_allreduce=args.root_allreduce)
    else:
        apply_fsdp(model, mesh)
        model.to_empty(device=torch.device("cuda", local))
    model.init_weights(seed=0)
    muon_names = set(model.muon_param_names())
    muon_p = [p for n, p in model.named_parameters() if n in muon_names]
    adam_p = [p for n, p in model.named_parameters() if n not in muon_names]
    opts = [MuonOptimizer(muon_p, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=False, ns_steps=5),
            FusedAdamW(adam_p, lr=1e-3, weight_decay=0.01)]
    if ctl is not None:
        for o in opts:
            ctl.attach_optimizer(o)
    return model, opts, cfg.vocab_size


def launch_counter():
    from my_muon_fsdp2_b200._ext import launch_count

    return launch_count


# ------------------------------------------------------------------------ reference arm
def build_reference(args, world, local):
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "muon_fsdp")):
        raise RuntimeError("reference package not installed under baseline/_ref")
    sys.path.insert(0, ref)
    import muon_fsdp  # noqa: F401  (the unmodified reference)
    from muon_fsdp import MuonOptimizer as RefMuon
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import fully_shard
    from transformers import LlamaConfig as HFConfig
    from transformers import LlamaForCausalLM

    hf = HFConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=args.layers,
                  num_attention_heads=32, num_key_value_heads=8, rope_theta=500000.0, max_position_embeddings=8192,
                  rms_norm_eps=1e-5, tie_word_embeddings=False, attn_implementation="sdpa", use_cache=False)
    mesh = init_device_mesh("cuda", (world,))
    with torch.device("meta"):
        model = LlamaForCausalLM(hf).to(torch.bfloat16)
    for layer in model.model.layers:
        fully_shard(layer, mesh=mesh)
    fully_shard(model, mesh=mesh)
    model.to_empty(device=torch.device("cuda", local))
    with torch.no_grad():
        for n, p in model.named_parameters():
            loc = p.to_local()
            if "norm" in n:
                loc.fill_(1.0)
            else:
                loc.normal_(0.0, 0.02)
    muon_p = [p for n, p in model.named_parameters() if p.dim() == 2 and (".self_attn." in n or ".mlp." in n)]
    ids = {id(p) for p in muon_p}
    adam_p = [p for p in model.parameters() if id(p) not in ids]
    opts = [RefMuon(muon_p, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=False, ns_steps=5),
            torch.optim.AdamW(adam_p, lr=1e-3, weight_decay=0.01)]
    return model, opts, hf.vocab_size


class RefTrainer:
    """The reference has no trainer API for this model; its examples' loop (train_gpt.py:330-383)."""

    def __init__(self, model, opts, ga, step_timer=None):
        self.model, self.opts, self.ga, self.step_timer = model, opts, ga, step_timer

    def step_on_device(self, tokens):
        total = None
        for i in range(self.ga):
            self.model.set_requires_gradient_sync(i == self.ga - 1)
            t = tokens[i]
            loss = self.model(input_ids=t[:, :-1], labels=t[:, :-1]).loss / self.ga
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
        if self.step_timer is not None:
            self.step_timer.start()
        for o in self.opts:
            o.step()
        if self.step_timer is not None:
            self.step_timer.stop()
        for o in self.opts:
            o.zero_grad(set_to_none=True)
        return total

    def train_step(self, batch):
        return float(self.step_on_device(batch.to("cuda", non_blocking=True)).item())


# ---------------------------------------------------------------------------------- main
def main():
    args = parse()
    rank, world, local = init_dist()
    from my_muon_fsdp2_b200.utils.clocks import ClockSampler, physical_gpu_index
    from my_muon_fsdp2_b200.utils.timing import EventTimer, max_over_ranks

    ga, mbs, seq = args.grad_accum, args.micro_bs, args.seq
    tokens_per_step = world * ga * mbs * seq
    try:
        if args.impl == "reference":
            model, opts, vocab = build_reference(args, world, local)
            count = None
        else:
            model, opts, vocab = build_ours(args, world, local)
            count = launch_counter()
    except Exception as e:  # reference cannot be built/installed: say so in one line
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"[:300]}))
            dist.destroy_process_group()
            return
        raise
    opt_timer = EventTimer()
    if args.impl == "reference":
        trainer = RefTrainer(model, opts, ga, step_timer=opt_timer)
    else:
        from my_muon_fsdp2_b200.train import Trainer

        trainer = Trainer(model, opts, grad_accum=ga, step_timer=opt_timer, keep_gathered=args.keep_gathered,
                          time_phases=not args.no_phases)

    dev_batches = [synthetic_tokens(s, ga, mbs, seq, vocab, rank, device="cuda") for s in range(2)]
    warmup, steps, e2e_cap, settle = args.warmup, args.steps, 3, True
    budget = None
    t_begin = time.time()
    s = 0
    while s < warmup:
        t0 = time.time()
        trainer.step_on_device(dev_batches[s % 2])
        torch.cuda.synchronize()
        s += 1
        if args.impl == "reference" and s == 2 and args.ref_budget_s > 0:
            # the reference's steps take tens of seconds (fp32 larger-Gram Newton-Schulz on every
            # rank): fit the run into the wall-clock budget, with fewer timed steps if needed.  Every
            # rank takes the same decision (slowest rank's step time).
            t_step = torch.tensor([time.time() - t0], dtype=torch.float64, device="cuda")
            dist.all_reduce(t_step, op=dist.ReduceOp.MAX)
            t_step = float(t_step.item())
            elapsed = time.time() - t_begin
            planned = elapsed + (warmup - 2 + steps + min(steps, 3) + 1) * t_step
            if planned > args.ref_budget_s:
                warmup = max(3, s)
                left = args.ref_budget_s - elapsed - (warmup - s) * t_step
                steps = max(1, min(args.steps, int(left / t_step) - 1))
                e2e_cap, settle = 1, False
                budget = {"budget_s": args.ref_budget_s, "step_s_estimate": t_step, "steps_requested": args.steps,
                          "warmup_requested": args.warmup}
    torch.cuda.synchronize()
    if args.impl == "ours":
        from my_muon_fsdp2_b200._ext import check_device_error

        check_device_error(local)
    opt_timer.pairs.clear()
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    n0 = count() if count else 0
    mem0 = torch.cuda.memory_stats()
    # one event per step boundary (recording an event adds no work between the steps)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    start, end = marks[0], marks[-1]
    start.record()
    step_marks, host_marks, probes = [], [], []
    host_t0 = time.perf_counter()
    for s in range(steps):
        loss = trainer.step_on_device(dev_batches[s % 2])
        marks[s + 1].record()
        step_marks.append(list(getattr(trainer, "_phase_marks", [])))  # read after the loop
        host_marks.append(list(getattr(trainer, "_host_marks", [])))
        probes.append(list(getattr(trainer, "_probes", [])))
    host_loop_ms = (time.perf_counter() - host_t0) * 1e3 / steps  # host time to enqueue one step
    torch.cuda.synchronize()
    phase_sum: dict = {}
    for pm in step_marks:
        for (_, a), (name, b) in zip(pm[:-1], pm[1:]):
            phase_sum[name] = phase_sum.get(name, 0.0) + a.elapsed_time(b)
    launches = (count() - n0) if count else None
    mem1 = torch.cuda.memory_stats()
    # device memory of this rank, and what the caching allocator had to do inside the timed steps
    # (cudaMalloc calls, and retries that free cached blocks, which synchronise the device)
    memory = {"max_reserved_gb": round(mem1.get("reserved_bytes.all.peak", 0) / 2**30, 2),
              "max_allocated_gb": round(mem1.get("allocated_bytes.all.peak", 0) / 2**30, 2),
              "timed_cuda_mallocs": mem1.get("num_device_alloc", 0) - mem0.get("num_device_alloc", 0),
              "timed_alloc_retries": mem1.get("num_alloc_retries", 0) - mem0.get("num_alloc_retries", 0)}
    clk = clocks.stop()
    dist.barrier()
    dev_ms = max_over_ranks(start.elapsed_time(end) / steps)
    # per-step spread (each step's max over ranks), so that a few-percent change between runs
    # can be told apart from step-to-step noise
    per_step = [max_over_ranks(marks[i].elapsed_time(marks[i + 1])) for i in range(steps)]
    srt = sorted(per_step)
    spread = {"min": srt[0], "median": srt[len(srt) // 2], "max": srt[-1]}
    phases = {k: max_over_ranks(v / steps) for k, v in sorted(phase_sum.items())} if phase_sum else None
    host_sum: dict = {}
    for hm in host_marks:
        for (_, a), (name, b) in zip(hm[:-1], hm[1:]):
            host_sum[name] = host_sum.get(name, 0.0) + (b - a) * 1e3
    host_phases = {k: round(v / steps, 2) for k, v in sorted(host_sum.items())} if host_sum else None
    clock_at = {}  # MMF_CLOCK_PROBE=1: mean SM MHz measured at the end of each phase
    for pr in probes:
        for name, t in pr:
            v = t.double()
            clock_at.setdefault(name, []).append(float((v[:, 0] / v[:, 1]).mean()) * 1e3)
    clock_at = {k: round(sum(v) / len(v), 1) for k, v in clock_at.items()}
    opt_ms = max_over_ranks(opt_timer.mean_ms())
    final_loss = float(loss.item())

    e2e = None
    if not args.no_e2e:
        host = [synthetic_tokens(100 + s, ga, mbs, seq, vocab, rank).pin_memory() for s in range(2)]
        if settle:
            trainer.train_step(host[0])
        torch.cuda.synchronize()
        dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        # at most 3 timed end-to-end steps: the reference arm's steps take about a minute each
        # at 32 layers (its fp32 larger-Gram Newton-Schulz), and both arms use the same count
        e2e_steps = min(steps, e2e_cap)
        t0.record()
        for s in range(e2e_steps):
            trainer.train_step(host[s % 2])
        t1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(t0.elapsed_time(t1) / e2e_steps)
        e2e = {"value": tokens_per_step / (e2e_ms / 1e3), "unit": "tokens/s", "steps": e2e_steps,
               "h2d_bytes_per_step": host[0].numel() * host[0].element_size(), "d2h_bytes_per_step": 4,
               "ms_per_step": e2e_ms, "api": ("my_muon_fsdp2_b200.train.Trainer.train_step" if args.impl == "ours"
                                               else "reference example loop (no trainer API in the reference)")}

    if rank == 0:
        value = tokens_per_step / (dev_ms / 1e3)
        base = baseline_value()
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, **({"wall_clock_budget": budget} if budget else {}), "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / base) if base else None, "dtype": "bf16",
            "data": "synthetic uniform random tokens; random-init weights",
            "optimizer_step_ms": opt_ms, "step_ms_spread": spread,
            **({"phase_ms": phases} if phases else {}),
            **({"host_phase_ms": host_phases, "host_enqueue_ms_per_step": round(host_loop_ms, 1)}
               if host_phases else {}),
            **({"sm_mhz_after_phase": clock_at} if clock_at else {}),
            "config": {"model": MODEL_DESC if args.layers == 32 else f"{MODEL_DESC} [DEBUG: {args.layers} layers]",
                       "global_batch": world * ga * mbs, "seq_len": seq, "grad_accum": ga,
                       "micro_batch_per_gpu": mbs, "parallelism": f"fsdp{world}",
                       "root_params": ("fully_shard" if (args.impl == "reference" or args.fsdp != "symm"
                                                         or (world > 1 and args.root == "shard"))
                                       else "replicated, one gradient all-reduce per step" if world > 1
                                       else "unsharded (one rank)"),
                       "fsdp_impl": ((args.fsdp + (f"/{args.rs_mode}" if args.fsdp == "symm" else "")
                                      + ("/keep_gathered" if args.keep_gathered else ""))
                                     if args.impl == "ours" else "fully_shard"),
                       "tokens_per_step": tokens_per_step,
                       "l2": "no flush: per-step working set (16 GB bf16 weights + activations) >> 126 MB L2",
                       "optimizers": "Muon(attn+FFN matrices, lr .02, mom .95, wd .01, ns 5) + AdamW(rest, lr 1e-3)"},
            "clocks": clk, "e2e": e2e, "gpu_launches": launches, "final_loss": final_loss, "memory": memory,
        }
        if args.impl == "reference":
            out["impl"] = "reference"
        print(json.dumps(out))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
