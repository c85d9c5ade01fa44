"""Real sharded semantics on CPU gloo ranks: FSDP2 (fully_shard) + our optimizers must give the
same parameters as a single-process run (the reference never compares across world sizes)."""
import copy

import pytest
import torch
import torch.nn as nn

from tests.conftest import rel_err
from tests.dist_util import run_ranks

pytestmark = pytest.mark.distributed


def _mlp(seed=0, d_in=512, hidden=2048, d_out=512):
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(d_in, hidden), nn.GELU(), nn.Linear(hidden, d_out))


def _data(step, d_in=512, d_out=512, batch=64):
    g = torch.Generator().manual_seed(1000 + step)
    return torch.randn(batch, d_in, generator=g), torch.randn(batch, d_out, generator=g)


def _train(model, opt, steps, d_in, d_out):
    losses = []
    for s in range(steps):
        x, y = _data(s, d_in, d_out)
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


def _make_opt(kind, model):
    from my_muon_fsdp2_b200 import FSDPMuonOptimizer, MuonOptimizer
    from my_muon_fsdp2_b200.fsdp2_utils import MuonOptimizer as ModelMuon

    if kind == "fsdp":
        return FSDPMuonOptimizer(model, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True, ns_steps=5)
    if kind == "muon":
        return MuonOptimizer(model.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True)
    if kind == "model_muon":
        return ModelMuon(model, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True)
    if kind == "sso":
        from my_muon_fsdp2_b200 import SpectralSphereOptimizer

        torch.manual_seed(11)  # the power iteration's start vector: the same on every rank
        return SpectralSphereOptimizer(model.parameters(), lr=0.02, momentum=0.95, power_iteration_steps=20)
    if kind == "hybrid":
        from my_muon_fsdp2_b200 import create_hybrid_optimizer

        return create_hybrid_optimizer(model, muon_lr=0.02, adamw_lr=1e-3, muon_weight_decay=0.01)
    raise ValueError(kind)


def _sharded_worker(rank, world, kind, steps, dims):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import fully_shard

    d_in, hidden, d_out = dims
    model = _mlp(0, d_in, hidden, d_out)
    mesh = init_device_mesh("cpu", (world,))
    for m in model:
        if isinstance(m, nn.Linear):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    opt = _make_opt(kind, model)
    losses = _train(model, opt, steps, d_in, d_out)
    full = [p.full_tensor().detach().clone() for p in model.parameters()]
    return {"losses": losses, "params": full}


@pytest.mark.parametrize("kind", ["fsdp", "muon", "model_muon", "sso", "hybrid"])
def test_sharded_equals_single_process(kind):
    """The CPU/gloo MLP workload (512->2048->512, world size 2), shortened to 6 steps."""
    dims, steps = (512, 2048, 512), 6
    res = run_ranks(_sharded_worker, 2, kind, steps, dims)
    model = _mlp(0, *dims)
    opt = _make_opt(kind, model)
    losses = _train(model, opt, steps, dims[0], dims[2])
    for a, b in zip(res["losses"], losses):
        assert abs(a - b) < 1e-4 * max(1.0, abs(b))
    for p, q in zip(res["params"], model.parameters()):
        assert rel_err(p, q.detach()) < 1e-4


def test_uneven_rows_three_ranks():
    """Rows not divisible by the world size follow torch.chunk sharding (the reference raises)."""
    dims, steps = (24, 37, 11), 3
    res = run_ranks(_sharded_worker, 3, "fsdp", steps, dims)
    model = _mlp(0, *dims)
    opt = _make_opt("fsdp", model)
    _train(model, opt, steps, dims[0], dims[2])
    for p, q in zip(res["params"], model.parameters()):
        assert rel_err(p, q.detach()) < 1e-4


def _collectives_worker(rank, world):
    from my_muon_fsdp2_b200.fsdp2_utils import (all_gather, all_reduce_avg, all_reduce_sum, broadcast, get_rank,
                                                get_world_size, scatter, scatter_updates)

    out = {}
    t = torch.full((2, 3), float(rank))
    out["gather"] = all_gather([t, torch.arange(4.0) + rank])
    out["sum"] = all_reduce_sum(torch.tensor([1.0 + rank]))
    out["avg"] = all_reduce_avg(torch.tensor([1.0 + rank]))
    out["bcast"] = broadcast(torch.tensor([float(rank)]), src=1)
    out["scatter"] = scatter([torch.arange(8.0).view(4, 2)])[0]
    out["scatter_updates"] = scatter_updates([torch.arange(6.0).view(3, 2)])[0]
    out["ws"] = (get_rank(), get_world_size())
    return out


def test_collectives_gloo():
    out = run_ranks(_collectives_worker, 2)
    g, v = out["gather"]
    assert g.shape == (4, 3) and torch.equal(g[:2], torch.zeros(2, 3)) and torch.equal(g[2:], torch.ones(2, 3))
    assert torch.equal(v, torch.cat([torch.arange(4.0), torch.arange(4.0) + 1]))
    assert out["sum"].item() == 3.0 and out["avg"].item() == 1.5 and out["bcast"].item() == 1.0
    assert torch.equal(out["scatter"], torch.arange(4.0).view(2, 2))
    assert torch.equal(out["scatter_updates"], torch.arange(4.0).view(2, 2))  # torch.chunk: rows 0-1 on rank 0
    assert out["ws"] == (0, 2)


def _hsdp_worker(rank, world):
    from torch.distributed.fsdp import fully_shard

    from my_muon_fsdp2_b200 import HDSPMuonOptimizer, create_device_mesh_2d, get_hsdp_groups

    mesh = create_device_mesh_2d(2, 2)
    dpg, fg = get_hsdp_groups(mesh)
    model = _mlp(0, 16, 40, 8)
    for m in model:
        if isinstance(m, nn.Linear):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    opt = HDSPMuonOptimizer(model, device_mesh=mesh, lr=0.01)
    losses = _train(model, opt, 3, 16, 8)
    return {"losses": losses, "params": [p.full_tensor().detach().clone() for p in model.parameters()],
            "groups": (torch.distributed.get_world_size(dpg), torch.distributed.get_world_size(fg))}


def test_hsdp_2x2_matches_single_process():
    from my_muon_fsdp2_b200 import HDSPMuonOptimizer

    res = run_ranks(_hsdp_worker, 4)
    assert res["groups"] == (2, 2)
    model = _mlp(0, 16, 40, 8)
    opt = HDSPMuonOptimizer(model, lr=0.01)
    _train(model, opt, 3, 16, 8)
    for p, q in zip(res["params"], model.parameters()):
        assert rel_err(p, q.detach()) < 1e-4


def _scaled_worker(rank, world, use_scaler):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import fully_shard
    from torch.distributed.fsdp.sharded_grad_scaler import ShardedGradScaler

    from my_muon_fsdp2_b200 import MuonOptimizer

    model = _mlp(0, 64, 128, 32)
    mesh = init_device_mesh("cpu", (world,))
    for m in model:
        if isinstance(m, nn.Linear):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    opt = MuonOptimizer(model.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01)
    scaler = ShardedGradScaler(device="cpu", init_scale=256.0) if use_scaler else None
    for s in range(2):
        x, y = _data(s, 64, 32, batch=8)
        opt.zero_grad()
        loss = ((model(x) - y) ** 2).mean()
        if scaler is None:
            loss.backward()
            opt.step()
        else:
            scaler.scale(loss).backward()
            scaler.step(opt)
            scaler.update()
    return [p.full_tensor().detach().clone() for p in model.parameters()]


def test_sharded_grad_scaler_with_fsdp2():
    """The reference trainer's FSDP + AMP recipe (ShardedGradScaler, train_gpt.py:324,343)
    drives the sharded Muon step like an unscaled one."""
    plain = run_ranks(_scaled_worker, 2, False)
    scaled = run_ranks(_scaled_worker, 2, True)
    for p, q in zip(scaled, plain):
        assert rel_err(p, q) < 1e-5
