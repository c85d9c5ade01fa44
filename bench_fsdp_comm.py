"""FSDP collectives of one Llama-3-8B block's linears, fused kernels vs NCCL + cuBLAS.

For each weight W [N, K] (row-sharded over the ranks) and T tokens per rank:
  * forward  : NCCL all_gather_into_tensor(W) + F.linear     vs  ag_gemm (one kernel)
  * weight-gradient: dY^T X (cuBLAS) + NCCL reduce_scatter_tensor(avg)  vs the SymmFSDP path of
                     --rs-mode: "fused" = wgrad_scatter (the GEMM epilogue stores each owner's rows
                     over NVLink) + side-stream barrier + rs_reduce; "overlap" = local GEMM +
                     side-stream barrier + rs_pull_reduce (both joined before the end event)
CUDA events on the launching stream, max over ranks, after warm-up; inputs are larger than L2
for the big shapes (weights 32-117 MB bf16, activations 32-117 MB).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench_fsdp_comm.py [--tokens 4096]
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

SHAPES = {"wq/wo": (4096, 4096), "wk/wv": (1024, 4096), "w1/w3": (14336, 4096), "w2": (4096, 14336)}


def timed(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def emulate(args, dev, ext, check_device_error, local):
    ws = args.emulate_world
    for name, (n, k) in SHAPES.items():
        if n % (128 * ws):
            continue
        w = torch.randn(n, k, device=dev, dtype=torch.bfloat16)
        x = torch.randn(args.tokens, k, device=dev, dtype=torch.bfloat16)
        g = torch.empty_like(w)
        ready = torch.zeros(n // 128 + 1, dtype=torch.int32, device=dev)
        ns = n // ws
        ptrs = [w.data_ptr() + 2 * s * ns * k for s in range(ws)]
        y = ext().ag_gemm(x, ptrs, 0, g, ready, 2e-3)
        torch.cuda.synchronize()
        ok = bool(torch.equal(g, w))
        ref = torch.nn.functional.linear(x, w)
        err = float((y.float() - ref.float()).norm() / ref.float().norm())
        t_ag = timed(lambda: ext().ag_gemm(x, ptrs, 0, g, ready, 2e-3), args.iters, args.warmup)
        t_mm = timed(lambda: torch.nn.functional.linear(x, w), args.iters, args.warmup)
        print(json.dumps({"metric": "ag_gemm emulated on one GPU (all shards local)", "weight": name, "N": n, "K": k,
                          "tokens": args.tokens, "emulated_world": ws, "ag_gemm_ms": t_ag, "cublas_ms": t_mm,
                          "gathered_equal": ok, "rel_err": err}))
    check_device_error(local)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--rs-mode", choices=["overlap", "fused"], default="overlap")
    ap.add_argument("--emulate-world", type=int, default=0,
                    help="one GPU: run ag_gemm as rank 0 of this many ranks whose shards are all local "
                         "buffers (the kernel's pull / ready-flag / GEMM structure without NVLink, for ncu)")
    args = ap.parse_args()
    if "RANK" not in os.environ:  # single process without torchrun
        import socket

        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from my_muon_fsdp2_b200._ext import check_device_error, ext
    from my_muon_fsdp2_b200.parallel.symm_fsdp import SymmFSDP


    T = args.tokens
    if args.emulate_world > 1:
        emulate(args, dev, ext, check_device_error, local)
        dist.destroy_process_group()
        return
    lins = {k: nn.Linear(kk, n, bias=False, device="meta") for k, (n, kk) in SHAPES.items()}
    for m in lins.values():
        m.to_empty(device=dev)
        m.to(torch.bfloat16)
        with torch.no_grad():
            m.weight.normal_(0, 0.02)
    names = list(lins)
    ctl = SymmFSDP([lins[k] for k in names], device=dev, rs_mode=args.rs_mode)
    rows = []
    for i, name in enumerate(names):
        n, k = SHAPES[name]
        x = torch.randn(T, k, device=dev, dtype=torch.bfloat16)
        dy = torch.randn(T, n, device=dev, dtype=torch.bfloat16)
        shard = ctl.params[i].to_local()
        full = torch.empty(n, k, device=dev, dtype=torch.bfloat16)

        def nccl_fwd():
            dist.all_gather_into_tensor(full, shard)
            return F.linear(x, full)

        def fused_fwd():
            ctl.valid[i] = False
            return ctl.linear_forward(i, x)

        rs_out = torch.empty(n // world, k, device=dev, dtype=torch.bfloat16)

        def nccl_wgrad():
            dw = dy.t() @ x
            dist.reduce_scatter_tensor(rs_out, dw, op=dist.ReduceOp.AVG)

        def fused_wgrad():
            ctl.params[i].grad = None
            ctl._accumulate_grad(i, dy, x)

        r = {"weight": name, "N": n, "K": k, "tokens": T, "rs_mode": args.rs_mode}
        r["fwd_nccl_ms"] = timed(nccl_fwd, args.iters, args.warmup)
        r["fwd_fused_ms"] = timed(fused_fwd, args.iters, args.warmup)
        r["gemm_only_ms"] = timed(lambda: F.linear(x, full), args.iters, args.warmup)
        r["wgrad_nccl_ms"] = timed(nccl_wgrad, args.iters, args.warmup)
        r["wgrad_fused_ms"] = timed(fused_wgrad, args.iters, args.warmup)
        r["wgrad_gemm_only_ms"] = timed(lambda: dy.t() @ x, args.iters, args.warmup)
        from my_muon_fsdp2_b200.ops.linear import mm_dw

        loc = torch.empty(n, k, device=dev, dtype=torch.bfloat16)
        r["wgrad_own_gemm_ms"] = timed(lambda: mm_dw([dy], x, [loc], False), args.iters, args.warmup)
        if args.rs_mode == "fused" and ctl.peer and ctl.fused_ok[i]:
            # the two halves of the fused path on their own: the GEMM whose epilogue stores each
            # owner's rows over NVLink, and the owner's rank-order sum of its region
            rr = ctl.rows[i]
            r["wgrad_scatter_only_ms"] = timed(lambda: ext().wgrad_scatter(dy, x, ctl._owner_ptrs[i], rr, None),
                                               args.iters, args.warmup)
            o = ctl.slot_offsets[i]
            region = ctl.slot_buf[o:o + world * rr * k]
            gsh = torch.empty(rr, k, device=dev, dtype=torch.bfloat16)
            r["rs_reduce_only_ms"] = timed(lambda: ext().rs_reduce(region, world, rr * k, gsh, False, 1.0 / world),
                                           args.iters, args.warmup)
        ref_dw = (dy.t() @ x).float()
        r["wgrad_own_rel_err"] = float((loc.float() - ref_dw).norm() / ref_dw.norm())
        # correctness spot check of the fused forward
        with torch.no_grad():
            y = fused_fwd()
            ref = F.linear(x, full)
        r["fwd_rel_err"] = float((y.float() - ref.float()).norm() / ref.float().norm())
        rows.append(r)
    torch.cuda.synchronize()
    check_device_error(local)
    if rank == 0:
        for r in rows:
            print(json.dumps({"metric": "fsdp collective + GEMM ms", "n_gpus": world, **r}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
