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


def engine_only(world, rank, local, comm):
    """One MuonEngine step on fixed DTensor shards of mixed shapes (incl. uneven rows and tall ones)."""
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard

    from my_muon_fsdp2_b200.parallel.muon_engine import MODE_EMA, MuonEngine, MuonHyper, MuonTask

    mesh = init_device_mesh("cuda", (world,))
    g = torch.Generator().manual_seed(7)
    shapes = [(512, 256), (256, 768), (300, 200), (1024, 256), (256, 1024), (96, 64)]
    out = {}
    params, tasks = [], []
    for i, (r, c) in enumerate(shapes):
        full_p = torch.randn(r, c, generator=g).to(torch.bfloat16)
        full_g = torch.randn(r, c, generator=g).to(torch.bfloat16)
        sh = lambda t: DTensor.from_local(t.chunk(world, 0)[rank].contiguous().to(f"cuda:{local}"), mesh, [Shard(0)],
                                          run_check=False, shape=t.shape, stride=t.stride())
        p = torch.nn.Parameter(sh(full_p))
        buf = torch.zeros(p.to_local().shape, dtype=torch.float32, device=f"cuda:{local}")
        tasks.append(MuonTask(param=p, grad=sh(full_g), buf=buf, lr_eff=0.05, decay=0.99))
        params.append(p)
    MuonEngine(comm=comm).step(tasks, MuonHyper(mode=MODE_EMA, momentum=0.9, nesterov=True))
    torch.cuda.synchronize()
    return {i: p.full_tensor().float().cpu() for i, p in enumerate(params)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="nccl")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--out", required=True)
    ap.add_argument("--engine-only", action="store_true")
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    if a.engine_only:
        res = engine_only(world, rank, local, a.comm)
        from my_muon_fsdp2_b200._ext import check_device_error

        check_device_error(local)
        if rank == 0:
            torch.save(res, a.out)
        dist.barrier()
        dist.destroy_process_group()
        return
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
