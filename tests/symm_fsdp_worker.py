"""Worker for the multi-GPU SymmFSDP tests (launched with torchrun by tests/test_gpu_symm_fsdp.py).

``--mode kernels``: fused all-gather GEMM and GEMM -> reduce-scatter on single linears, checked
against fp32 references built from all ranks' inputs.  ``--mode train``: a small Llama trained
for a few steps with SymmFSDP linears and with plain FSDP2; rank 0 saves both trajectories."""
import argparse
import datetime
import os

import torch
import torch.distributed as dist
import torch.nn as nn


def _gather(t):
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return parts


def run_kernels(rank, world, dev):
    from my_muon_fsdp2_b200._ext import check_device_error
    from my_muon_fsdp2_b200.parallel.symm_fsdp import SymmFSDP

    shapes = [(1024, 512), (512, 1024), (256 * world, 256), (768 * world, 512)]
    res = {}
    for mode in ("overlap", "fused"):
        torch.manual_seed(0)
        lins = [nn.Linear(k, n, bias=False).to(dev, torch.bfloat16) for n, k in shapes]
        fulls = [m.weight.detach().clone() for m in lins]
        ctl = SymmFSDP(lins, device=dev, rs_mode=mode)
        assert ctl.fused
        _check_linears(ctl, lins, fulls, rank, world, dev, res, mode)
    torch.cuda.synchronize()
    check_device_error(dev.index)
    return res


def run_mixed(rank, world, dev):
    """A weight the fused kernels take next to one they do not (NCCL path), both with biases."""
    from my_muon_fsdp2_b200._ext import check_device_error
    from my_muon_fsdp2_b200.parallel.symm_fsdp import SymmFSDP

    res = {}
    torch.manual_seed(0)
    lins = [nn.Linear(512, 256 * world).to(dev, torch.bfloat16), nn.Linear(512, 192 * world).to(dev, torch.bfloat16)]
    fulls = [m.weight.detach().clone() for m in lins]
    ctl = SymmFSDP(lins, device=dev)
    res["fused_ok"] = list(ctl.fused_ok)
    _check_linears(ctl, lins, fulls, rank, world, dev, res, "mixed")
    torch.cuda.synchronize()
    check_device_error(dev.index)
    return res


def _check_linears(ctl, lins, fulls, rank, world, dev, res, mode):
    for i, (m, w) in enumerate(zip(lins, fulls)):
        for t in (256, 200):  # 200: token count padded to the tile size inside
            g = torch.Generator(device="cpu").manual_seed(1000 * i + 10 * rank + t)
            x = torch.randn(t, w.shape[1], generator=g).to(dev, torch.bfloat16).requires_grad_(True)
            ctl.invalidate()
            m.weight.grad = None
            y = m(x)  # fused all-gather GEMM
            y2 = m(x)  # resident full weight
            ref = x.detach().float() @ w.float().t()
            if m.bias is not None:
                ref = ref + m.bias.detach().float()
            res[f"y{i}_{t}_{mode}"] = ((y.float() - ref).norm() / ref.norm()).item()
            res[f"y2{i}_{t}_{mode}"] = ((y2.float() - ref).norm() / ref.norm()).item()
            res[f"g{i}_{t}_{mode}"] = bool(torch.equal(ctl.full[i], w))
            dy = torch.randn(t, w.shape[0], generator=g).to(dev, torch.bfloat16)
            y.backward(dy)
            xs, dys = _gather(x.detach()), _gather(dy)
            dw = sum(d.float().t() @ a.float() for d, a in zip(dys, xs)) / world
            r = w.shape[0] // world
            dw_loc = dw[rank * r:(rank + 1) * r]
            got = m.weight.grad.to_local().float()
            res[f"dw{i}_{t}_{mode}"] = ((got - dw_loc).norm() / dw_loc.norm()).item()
            dx_ref = dy.float() @ w.float()
            res[f"dx{i}_{t}_{mode}"] = ((x.grad.float() - dx_ref).norm() / dx_ref.norm()).item()


def run_hsdp(rank, world, dev):
    """2 x (world / 2) mesh (replicate, shard): SymmFSDP HSDP against FSDP2 HSDP."""
    return run_train(rank, world, dev, mesh_shape=(2, world // 2))


def run_train_shard_root(rank, world, dev):
    """The same comparison with the rest of the model under FSDP2 instead of replicated."""
    return run_train(rank, world, dev, root="shard")


def run_train(rank, world, dev, steps=3, mesh_shape=None, root="replicate"):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import FusedAdamW, MuonOptimizer
    from my_muon_fsdp2_b200.models.llama import Llama, LlamaConfig, apply_fsdp
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    out = {}
    for mode in ("symm", "fsdp2"):
        torch.manual_seed(0)
        cfg = LlamaConfig.tiny(dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024, vocab_size=1024, n_layers=2)
        model = Llama(cfg).to(dev, torch.bfloat16)
        if mesh_shape:  # (replicate, shard): FSDP2's HSDP wants the dimensions named
            mesh = init_device_mesh("cuda", mesh_shape, mesh_dim_names=("dp_replicate", "fsdp_shard"))
        else:
            mesh = init_device_mesh("cuda", (world,))
        if mode == "symm":
            ctl = apply_symm_fsdp(model, mesh, root=root)
        else:
            apply_fsdp(model, mesh)
        names = set(model.muon_param_names())
        opts = [MuonOptimizer([p for n, p in model.named_parameters() if n in names], lr=0.02, weight_decay=0.01),
                FusedAdamW([p for n, p in model.named_parameters() if n not in names], lr=1e-3)]
        if mode == "symm":
            for o in opts:
                ctl.attach_optimizer(o)
        losses = []
        for s in range(steps):
            g = torch.Generator().manual_seed(100 * s + rank)
            tok = torch.randint(0, cfg.vocab_size, (2, 2, 129), generator=g).to(dev)
            tot = 0.0
            for mb in range(2):
                model.set_requires_gradient_sync(mb == 1)
                loss = model(tok[mb, :, :-1], tok[mb, :, 1:]) / 2
                loss.backward()
                tot += loss.item()
            for o in opts:
                o.step()
                o.zero_grad(set_to_none=True)
            losses.append(tot)
        params = {n: (p.full_tensor() if hasattr(p, "full_tensor") else p).detach().float().cpu()
                  for n, p in model.named_parameters()}
        # matrices whose owner wrote the update straight into every rank's parameter shard
        direct = float(opts[0]._engine.last_stats.get("direct_updates", 0.0))
        out[mode] = {"losses": losses, "params": params, "direct_updates": direct}
        del model, opts
        torch.cuda.synchronize()
    return out


def run_split(rank, world, dev, steps=2):
    """Muon with the cooperative all-rank chain vs owner-computes on the same FSDP2 model."""
    from torch.distributed.fsdp import fully_shard

    from my_muon_fsdp2_b200 import MuonOptimizer

    out = {}
    for schedule in ("always", "never"):
        torch.manual_seed(0)
        model = nn.Sequential(nn.Linear(2048, 512, bias=False), nn.Linear(1024, 1024, bias=False)).to(dev)
        for m in model:
            fully_shard(m)
        fully_shard(model)
        opt = MuonOptimizer(model.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01, schedule=schedule)
        for s in range(steps):
            g = torch.Generator(device="cpu").manual_seed(s)
            for p in model.parameters():
                p.grad = None
            w0, w1 = model[0].weight, model[1].weight
            # synthetic gradients (the same full matrices on every rank, sharded like the params)
            from torch.distributed.tensor import distribute_tensor

            for w in (w0, w1):
                full = torch.randn(w.shape, generator=g).to(dev)
                w.grad = distribute_tensor(full, w.device_mesh, w.placements)
            opt.step()
            assert opt._engine.split_count == (2 if schedule == "always" else 0)
        out[schedule] = {n: p.full_tensor().detach().float().cpu() for n, p in model.named_parameters()}
    torch.cuda.synchronize()
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(dev.index)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["kernels", "train", "train_shard_root", "split", "mixed", "hsdp"],
                    required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    try:
        res = {"kernels": run_kernels, "train": run_train, "train_shard_root": run_train_shard_root,
               "split": run_split, "mixed": run_mixed, "hsdp": run_hsdp}[a.mode](
            rank, world, dev)
        if rank == 0:
            torch.save(res, a.out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
