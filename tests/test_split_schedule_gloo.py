"""Cooperative (all-rank) Newton–Schulz schedule: the per-shape selector, and sharded results on
gloo ranks equal to a single-process Muon step."""
import pytest
import torch
import torch.nn as nn

from tests.conftest import rel_err
from tests.dist_util import run_ranks


def test_selector_splits_only_dominant_matrices():
    from my_muon_fsdp2_b200.parallel.muon_engine import select_split, split_eligible

    sweep = [(4096, 4096), (1024, 4096), (4096, 14336), (14336, 4096), (8192, 28672)]
    for w in (2, 4, 8):
        assert select_split(sweep, w, 5) == [4]
    llama = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
             (4096, 14336)] * 32
    assert select_split(llama, 8, 5) == []
    assert not split_eligible(14336, 4096, 2)  # tall: owner-computes only
    assert not split_eligible(8192, 28672, 1)
    assert not split_eligible(8192 + 128, 28672, 8)


def _model():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(1024, 512, bias=False), nn.Linear(512, 512, bias=False))


def _data(step):
    g = torch.Generator().manual_seed(step)
    return torch.randn(32, 1024, generator=g), torch.randn(32, 512, generator=g)


def _sharded(rank, world, schedule, steps):
    from torch.distributed.fsdp import fully_shard

    from my_muon_fsdp2_b200 import MuonOptimizer

    model = _model()
    for m in model:
        fully_shard(m)
    fully_shard(model)
    opt = MuonOptimizer(model.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True,
                        schedule=schedule)
    for s in range(steps):
        x, y = _data(s)
        opt.zero_grad()
        ((model(x) - y) ** 2).mean().backward()
        opt.step()
        assert opt._engine.split_count == (2 if schedule == "always" else 0)
    return {n: p.full_tensor().detach().clone() for n, p in model.named_parameters()}


@pytest.mark.distributed
def test_cooperative_schedule_matches_single_process():
    from my_muon_fsdp2_b200 import MuonOptimizer

    steps = 3
    got = run_ranks(_sharded, 2, "always", steps)
    ref = _model()
    opt = MuonOptimizer(ref.parameters(), lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True)
    for s in range(steps):
        x, y = _data(s)
        opt.zero_grad()
        ((ref(x) - y) ** 2).mean().backward()
        opt.step()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.detach()) < 1e-4, n


def _peer_storage(rank, world):
    import torch.distributed as dist

    from my_muon_fsdp2_b200.parallel.symm import peer_param_addrs, register_peer_storage

    buf = torch.zeros(100)  # stands in for a symmetric buffer; the bases below are never dereferenced
    register_peer_storage(buf, dist.group.WORLD, [10_000, 20_000])
    out = {
        "inside": peer_param_addrs(buf[40:60].view(4, 5), dist.group.WORLD),
        "outside": peer_param_addrs(torch.zeros(4), dist.group.WORLD),
        "strided": peer_param_addrs(buf[:40].view(8, 5)[:, :2], dist.group.WORLD),
    }
    buf2 = torch.zeros(50, dtype=torch.bfloat16)  # a second store with its own bases
    register_peer_storage(buf2, dist.group.WORLD, [50_000, 60_000])
    out["second"] = peer_param_addrs(buf2[10:], dist.group.WORLD)
    sub = dist.new_group([0])
    if rank == 0:
        out["other_group"] = peer_param_addrs(buf[40:60], sub)
    return out


def test_peer_parameter_storage_addresses():
    """The Muon engine's in-place peer update finds every rank's copy of a parameter shard at
    the same offset of the registered symmetric buffer, and only for that buffer's group."""
    got = run_ranks(_peer_storage, 2)
    assert got["inside"] == [10_000 + 40 * 4, 20_000 + 40 * 4]
    assert got["outside"] is None and got["strided"] is None
    assert got["second"] == [50_000 + 10 * 2, 60_000 + 10 * 2]
    assert got["other_group"] is None
