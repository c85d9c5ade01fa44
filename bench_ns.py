"""Isolated Muon step sweep: gather + 5 quintic Newton–Schulz iterations + scatter-update.

Inputs: row-sharded (torch.chunk / FSDP2 Shard(0)) bf16 momentum matrices ~N(0,1), seeded;
shapes 4096x4096, 1024x4096, 4096x14336, 14336x4096, 8192x28672 (``--shapes`` to override).

* ``--impl ours``: the library's MuonEngine on DTensor shards (owner-computes schedule, fused
  momentum/NS/update kernels, ``--comm nccl|p2p`` exchange), one launch group per shape; the
  matrices that dominate the per-rank load (8192x28672) take the cooperative all-rank chain
  (``--schedule auto``; ``never``/``always`` force a schedule).
* ``--impl reference``: the reference's own path per matrix — ``muon_fsdp.distributed
  .all_gather_grads`` (NCCL all_gather_into_tensor) -> ``muon_fsdp.utils
  .zeropower_via_newtonschulz5`` (fp32, larger-side Gram) -> row slice -> ``add_``.

Each timed iteration processes every matrix once; CUDA events on the launching stream, max over
ranks.  Roofline per shape: max(FLOPs / measured bf16 GEMM peak, NVLink bytes / 770 GB/s).

    python bench_ns.py [--shapes 4096x14336,...] [--iters K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_ns.py ...
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_SHAPES = "4096x4096,1024x4096,4096x14336,14336x4096,8192x28672"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=DEFAULT_SHAPES)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--comm", choices=["auto", "nccl", "p2p"], default="auto")
    ap.add_argument("--ns-steps", type=int, default=5)
    ap.add_argument("--gemm-variant", type=int, default=0, help="0 auto, 1 single-CTA, 2 CTA pair")
    ap.add_argument("--repeat", type=int, default=1, help="every shape this many times (e.g. one per layer)")
    ap.add_argument("--schedule", choices=["auto", "never", "always"], default="auto",
                    help="cooperative all-rank NS chain per shape: auto (cost model), never, always")
    return ap.parse_args()


def init():
    if "RANK" not in os.environ:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["bf16_tflops"]) * 1e12, "measured"
    except Exception:
        return 1.59e15, "fallback"


def ns_flops_executed(m, n, steps):
    """FLOPs of the smaller-Gram chain (the work the math needs; SYRK halving not subtracted)."""
    a, b = min(m, n), max(m, n)
    return steps * (4.0 * a * a * b + 2.0 * a ** 3)


def main():
    args = parse()
    rank, world, local = init()
    dev = torch.device("cuda", local)
    shapes = [tuple(int(x) for x in s.split("x")) for s in args.shapes.split(",") if s] * args.repeat
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard

    mesh = init_device_mesh("cuda", (world,))
    g = torch.Generator(device="cpu").manual_seed(1234)
    by_shape = {}
    for r, c in shapes:  # one random matrix per distinct shape (repeats share values)
        if (r, c) not in by_shape:
            by_shape[(r, c)] = torch.randn(r, c, generator=g).to(torch.bfloat16)
    fulls = [by_shape[sh] for sh in shapes]

    def shard(t):
        return DTensor.from_local(t.chunk(world, 0)[rank].contiguous().to(dev), mesh, [Shard(0)], run_check=False,
                                  shape=t.shape, stride=t.stride())

    params = [torch.nn.Parameter(shard(torch.zeros_like(t))) for t in fulls]
    grads = [shard(t) for t in fulls]
    if args.impl == "ours":
        from my_muon_fsdp2_b200._ext import ext
        from my_muon_fsdp2_b200.parallel.muon_engine import MODE_COPY, MuonEngine, MuonHyper, MuonTask

        ext().set_gemm_variant(args.gemm_variant)

        engine = MuonEngine(comm=args.comm, split=args.schedule)
        hp = MuonHyper(mode=MODE_COPY, ns_steps=args.ns_steps)

        def step():
            tasks = [MuonTask(param=p, grad=gr, buf=None, lr_eff=0.02, decay=1.0) for p, gr in zip(params, grads)]
            engine.step(tasks, hp)
    else:
        sys.path.insert(0, os.path.join(HERE, "baseline", "_ref"))
        from muon_fsdp.distributed import all_gather_grads
        from muon_fsdp.utils import zeropower_via_newtonschulz5

        def step():
            full = all_gather_grads([gr.to_local() for gr in grads])
            for p, gf in zip(params, full):
                u = zeropower_via_newtonschulz5(gf, steps=args.ns_steps)
                rows = gf.shape[0] // world
                p.to_local().add_(u[rank * rows:(rank + 1) * rows], alpha=-0.02)

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    peak, src = peaks()
    flops = sum(ns_flops_executed(r, c, args.ns_steps) for r, c in shapes)
    nvl = sum(2 * 2 * r * c * (world - 1) / world for r, c in shapes) / world if world > 1 else 0.0
    roof_ms = max(flops / world / peak, nvl / 770e9) * 1e3
    if rank == 0:
        print(json.dumps({"metric": "isolated Muon step (gather+NS5+scatter-update) ms", "impl": args.impl,
                          "value": ms, "unit": "ms", "higher_is_better": False, "n_gpus": world,
                          "shapes": args.shapes, "repeat": args.repeat, "iters": args.iters, "warmup": args.warmup,
                          "tflops_effective": flops / (ms / 1e3) / 1e12,
                          "roofline_ms": roof_ms, "roofline_fraction": roof_ms / ms, "peak_source": src,
                          "comm": args.comm if args.impl == "ours" else "nccl all_gather",
                          "schedule": args.schedule if args.impl == "ours" else "replicated",
                          "cooperative_matrices": (engine.split_count if args.impl == "ours" else 0)}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
