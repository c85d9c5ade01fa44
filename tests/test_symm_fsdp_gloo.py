"""SymmFSDP semantics on CPU gloo ranks: the linears sharded by ``apply_symm_fsdp`` (collectives
through torch.distributed here; fused kernels on CUDA) must give the gradients and the training
trajectory of a single-process model trained on the union of the ranks' data."""
import copy

import pytest
import torch
import torch.nn as nn

from tests.conftest import rel_err
from tests.dist_util import run_ranks

pytestmark = pytest.mark.distributed

D, H = 256, 512


class Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.norm = nn.LayerNorm(D)
        self.up = nn.Linear(D, H, bias=False)
        self.down = nn.Linear(H, D, bias=False)

    def forward(self, x):
        return x + self.down(torch.nn.functional.gelu(self.up(self.norm(x))))


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.inp = nn.Linear(32, D)
        self.layers = nn.ModuleList([Block() for _ in range(2)])
        self.out = nn.Linear(D, 8)

    def forward(self, x):
        x = self.inp(x)
        for b in self.layers:
            x = b(x)
        return self.out(x)


def _data(step, rank, batch=16):
    g = torch.Generator().manual_seed(100 * step + rank)
    return torch.randn(batch, 32, generator=g), torch.randn(batch, 8, generator=g)


def _full(t):
    return t.full_tensor() if hasattr(t, "full_tensor") else t


def _symm_grads(rank, world, no_sync, root="shard"):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import SymmLinear, apply_symm_fsdp

    model = Net()
    ctl = apply_symm_fsdp(model, root=root)
    assert ctl.world == world and not ctl.fused
    assert sum(isinstance(m, SymmLinear) for m in model.modules()) == 4
    for step in range(2):  # two micro-batches: gradients accumulate
        if no_sync:
            model.set_requires_gradient_sync(step == 1)
        x, y = _data(step, rank)
        loss = ((model(x) - y) ** 2).mean() / 2
        loss.backward()
    from my_muon_fsdp2_b200.train.trainer import clip_grad_norm

    out = {n: _full(p.grad).clone() for n, p in model.named_parameters()}
    out["_norm"] = float(clip_grad_norm(list(model.parameters()), 1e9))  # norm only (no clipping)
    return out


@pytest.mark.parametrize("root", ["shard", "replicate"])
@pytest.mark.parametrize("no_sync", [False, True])
def test_symm_fsdp_grads_match_single_process(no_sync, root):
    """The rest of the model sharded by FSDP2 or replicated with one gradient all-reduce."""
    world = 2
    got = run_ranks(_symm_grads, world, no_sync, root)
    ref = Net()
    for step in range(2):
        xs, ys = zip(*[_data(step, r) for r in range(world)])
        loss = ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean() / 2
        loss.backward()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.grad) < 1e-5, n
    # the global gradient norm over sharded (DTensor) and replicated (plain) gradients
    ref_norm = float(torch.nn.utils.get_total_norm([p.grad for p in ref.parameters()], 2.0))
    assert abs(got["_norm"] - ref_norm) < 1e-5 * ref_norm


def _symm_train(rank, world, steps, root="shard", root_allreduce="hook"):
    from my_muon_fsdp2_b200 import MuonOptimizer
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = Net()
    if root == "replicate" and rank == 1:  # replicas start from rank 0's values
        with torch.no_grad():
            model.inp.weight.add_(1.0)
    ctl = apply_symm_fsdp(model, root=root, root_allreduce=root_allreduce)
    mats = [p for p in ctl.params]
    rest = [p for p in model.parameters() if all(p is not q for q in mats)]
    opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95, weight_decay=0.01), torch.optim.AdamW(rest, lr=1e-3)]
    for o in opts:
        ctl.attach_optimizer(o)
    losses = []
    for step in range(steps):
        x, y = _data(step, rank)
        loss = ((model(x) - y) ** 2).mean()
        loss.backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
        losses.append(loss.item())
    return {"params": {n: _full(p.detach()).clone() for n, p in model.named_parameters()}, "losses": losses}


@pytest.mark.parametrize("root,when", [("shard", "hook"), ("replicate", "hook"), ("replicate", "deferred")])
def test_symm_fsdp_training_matches_single_process(root, when):
    from my_muon_fsdp2_b200 import MuonOptimizer

    world, steps = 2, 3
    got = run_ranks(_symm_train, world, steps, root, when)
    ref = Net()
    mats = [m.weight for b in ref.layers for m in (b.up, b.down)]
    rest = [p for p in ref.parameters() if all(p is not q for q in mats)]
    opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95, weight_decay=0.01), torch.optim.AdamW(rest, lr=1e-3)]
    for step in range(steps):
        xs, ys = zip(*[_data(step, r) for r in range(world)])
        loss = ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean()
        loss.backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
    for n, p in ref.named_parameters():
        assert rel_err(got["params"][n], p.detach()) < 1e-4, n


class GatedBlock(nn.Module):
    """Two projections of the same input (as q/k/v or gate/up) through multi_linear."""

    def __init__(self):
        super().__init__()
        self.gate = nn.Linear(D, H, bias=False)
        self.up = nn.Linear(D, H, bias=False)
        self.down = nn.Linear(H, D, bias=False)

    def forward(self, x):
        from my_muon_fsdp2_b200.parallel.symm_fsdp import multi_linear

        g, u = multi_linear(x, (self.gate, self.up))
        return x + self.down(torch.nn.functional.silu(g) * u)


class GatedNet(nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(1)
        self.inp = nn.Linear(32, D)
        self.layers = nn.ModuleList([GatedBlock() for _ in range(2)])
        self.out = nn.Linear(D, 8)

    def forward(self, x):
        x = self.inp(x)
        for b in self.layers:
            x = b(x)
        return self.out(x)


def _gated_grads(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = GatedNet()
    apply_symm_fsdp(model)
    for step in range(2):
        model.set_requires_gradient_sync(step == 1)
        x, y = _data(step, rank)
        ((model(x) - y) ** 2).mean().div(2).backward()
    return {n: _full(p.grad).clone() for n, p in model.named_parameters()}


def test_symm_fsdp_multi_linear_grads_match_single_process():
    got = run_ranks(_gated_grads, 2)
    ref = GatedNet()
    for step in range(2):
        xs, ys = zip(*[_data(step, r) for r in range(2)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.grad) < 1e-5, n


def _ckpt_roundtrip(rank, world, path):
    from my_muon_fsdp2_b200 import MuonOptimizer
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp
    from my_muon_fsdp2_b200.train import load_checkpoint, save_checkpoint

    model = Net()
    ctl = apply_symm_fsdp(model)
    opt = MuonOptimizer(list(ctl.params), lr=0.02, momentum=0.95)
    ctl.attach_optimizer(opt)
    x, y = _data(0, rank)
    ((model(x) - y) ** 2).mean().backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    save_checkpoint(path, "net", model, opt, epoch=1, loss=0.0)
    ref_out = model(x).detach()

    torch.manual_seed(123)  # different init: the checkpoint must overwrite it
    fresh = Net()
    for p in fresh.parameters():
        torch.nn.init.normal_(p)
    ctl2 = apply_symm_fsdp(fresh)
    opt2 = MuonOptimizer(list(ctl2.params), lr=0.02, momentum=0.95)
    fresh(x)  # gathers the pre-load weights, which the load must invalidate
    meta = load_checkpoint(f"{path}/muon_net.pt", fresh, opt2)
    out = fresh(x).detach()
    return {"ref": ref_out, "out": out, "epoch": meta["epoch"]}


def test_symm_fsdp_checkpoint_roundtrip(tmp_path):
    got = run_ranks(_ckpt_roundtrip, 2, str(tmp_path))
    assert got["epoch"] == 1
    assert rel_err(got["out"], got["ref"]) < 1e-6


class BiasBlock(nn.Module):
    def __init__(self):
        super().__init__()
        self.norm = nn.LayerNorm(D)
        self.up = nn.Linear(D, H)       # with bias
        self.down = nn.Linear(H, D)
        self.attn = nn.MultiheadAttention(D, 4, batch_first=True)  # its projections stay out

    def forward(self, x):
        h = self.norm(x)
        a, _ = self.attn(h[:, None], h[:, None], h[:, None])
        return x + a[:, 0] + self.down(torch.nn.functional.gelu(self.up(h)))


class BiasNet(nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(2)
        self.inp = nn.Linear(32, D)
        self.layers = nn.ModuleList([BiasBlock() for _ in range(2)])
        self.out = nn.Linear(D, 8)

    def forward(self, x):
        x = self.inp(x)
        for b in self.layers:
            x = b(x)
        return self.out(x)


def _bias_grads(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import SymmLinear, apply_symm_fsdp

    model = BiasNet()
    ctl = apply_symm_fsdp(model)
    assert len(ctl.params) == 4  # up/down of two blocks; the attention projections stay out
    assert not isinstance(model.layers[0].attn.out_proj, SymmLinear)
    for step in range(2):
        x, y = _data(step, rank)
        ((model(x) - y) ** 2).mean().div(2).backward()
    return {n: _full(p.grad).clone() for n, p in model.named_parameters()}


def test_symm_fsdp_biased_linears_match_single_process():
    got = run_ranks(_bias_grads, 2)
    ref = BiasNet()
    for step in range(2):
        xs, ys = zip(*[_data(step, r) for r in range(2)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.grad) < 1e-5, n


def _hsdp_run(rank, world, steps):
    """2 x 2 mesh (replicate, shard): weights sharded over pairs of ranks, replicated across
    the pairs; gradients reduce-scattered in the shard group, then averaged over replicas."""
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import MuonOptimizer
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("replicate", "shard"))
    model = Net()
    ctl = apply_symm_fsdp(model, mesh=mesh)
    assert ctl.world == 2 and ctl.replicas == 2
    assert ctl.rank == rank % 2
    assert [p.placements for p in ctl.params][0][0].is_replicate()
    # gradients of two micro-batches (the first without sync)
    for mb in range(2):
        model.set_requires_gradient_sync(mb == 1)
        x, y = _data(mb, rank)
        ((model(x) - y) ** 2).mean().div(2).backward()
    grads = {n: _full(p.grad).clone() for n, p in model.named_parameters()}
    for p in model.parameters():
        p.grad = None
    mats = list(ctl.params)
    rest = [p for p in model.parameters() if all(p is not q for q in mats)]
    opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95, weight_decay=0.01), torch.optim.AdamW(rest, lr=1e-3)]
    for o in opts:
        ctl.attach_optimizer(o)
    for step in range(steps):
        x, y = _data(10 + step, rank)
        ((model(x) - y) ** 2).mean().backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
    return {"grads": grads, "params": {n: _full(p.detach()).clone() for n, p in model.named_parameters()}}


def test_symm_fsdp_hsdp_mesh_matches_single_process():
    from my_muon_fsdp2_b200 import MuonOptimizer

    world, steps = 4, 2
    got = run_ranks(_hsdp_run, world, steps)
    ref = Net()
    for mb in range(2):
        xs, ys = zip(*[_data(mb, r) for r in range(world)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    for n, p in ref.named_parameters():
        assert rel_err(got["grads"][n], p.grad) < 1e-5, n
    ref.zero_grad(set_to_none=True)
    mats = [m.weight for b in ref.layers for m in (b.up, b.down)]
    rest = [p for p in ref.parameters() if all(p is not q for q in mats)]
    opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95, weight_decay=0.01), torch.optim.AdamW(rest, lr=1e-3)]
    for step in range(steps):
        xs, ys = zip(*[_data(10 + step, r) for r in range(world)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
    for n, p in ref.named_parameters():
        assert rel_err(got["params"][n], p.detach()) < 1e-4, n


def _traffic(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = Net()
    ctl = apply_symm_fsdp(model)
    x, y = _data(0, rank)
    for mb in range(2):
        model.set_requires_gradient_sync(mb == 1)
        ((model(x) - y) ** 2).mean().backward()
    return ctl.stats()


def test_symm_fsdp_traffic_counters():
    """One step of two micro-batches: each weight is gathered once and reduce-scattered once
    (the no-sync micro-batch moves nothing); counts are the other rank's shard bytes."""
    got = run_ranks(_traffic, 2)
    shard = sum((H // 2) * D + (D // 2) * H for _ in range(2)) * 4  # fp32, the other rank's rows
    assert got == {"bytes_gathered": shard, "bytes_reduced": shard, "bytes_replica": 0}


def _dcp_roundtrip(rank, world, path):
    """DCP sharded save / load with the fused-FSDP linears and FSDP2 for the rest: the resumed
    run's next step equals the uninterrupted run's."""
    from my_muon_fsdp2_b200 import MuonOptimizer
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp
    from my_muon_fsdp2_b200.train.checkpoint import load_sharded, save_sharded

    def build(seed_override=None):
        model = Net()
        if seed_override is not None:
            torch.manual_seed(seed_override)
            for p in model.parameters():
                torch.nn.init.normal_(p)
        ctl = apply_symm_fsdp(model)
        mats = list(ctl.params)
        rest = [p for p in model.parameters() if all(p is not q for q in mats)]
        opts = [MuonOptimizer(mats, lr=0.02, momentum=0.95), torch.optim.AdamW(rest, lr=1e-3)]
        for o in opts:
            ctl.attach_optimizer(o)
        return model, opts

    def step(model, opts, s):
        x, y = _data(s, rank)
        ((model(x) - y) ** 2).mean().backward()
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)

    model, opts = build()
    step(model, opts, 0)
    save_sharded(path, model, opts, extra={"step": 1})
    step(model, opts, 1)
    want = {n: _full(p.detach()).clone() for n, p in model.named_parameters()}

    model2, opts2 = build(seed_override=7)
    extra = load_sharded(path, model2, opts2)
    step(model2, opts2, 1)
    got = {n: _full(p.detach()).clone() for n, p in model2.named_parameters()}
    return {"extra": extra, "want": want, "got": got}


def test_symm_fsdp_dcp_checkpoint_resume(tmp_path):
    res = run_ranks(_dcp_roundtrip, 2, str(tmp_path / "ckpt"))
    assert res["extra"] == {"step": 1}
    for n in res["want"]:
        assert torch.equal(res["got"][n], res["want"][n]), n


class CkptNet(Net):
    """Net with each block under non-reentrant activation checkpointing."""

    def forward(self, x):
        from torch.utils.checkpoint import checkpoint

        x = self.inp(x)
        for b in self.layers:
            x = checkpoint(b, x, use_reentrant=False)
        return self.out(x)


def _ckpt_grads(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = CkptNet()
    apply_symm_fsdp(model)
    for mb in range(2):
        model.set_requires_gradient_sync(mb == 1)
        x, y = _data(mb, rank)
        ((model(x) - y) ** 2).mean().div(2).backward()
    return {n: _full(p.grad).clone() for n, p in model.named_parameters()}


def test_symm_fsdp_with_activation_checkpointing():
    """Recomputing a block in backward runs its SymmLinears' forward again (on the resident
    weights) and their gradient path once: gradients equal the single-process ones."""
    got = run_ranks(_ckpt_grads, 2)
    ref = Net()
    for mb in range(2):
        xs, ys = zip(*[_data(mb, r) for r in range(2)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.grad) < 1e-5, n


def _frozen(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = Net()
    model.layers[0].up.weight.requires_grad_(False)  # frozen before sharding
    ctl = apply_symm_fsdp(model)
    x, y = _data(0, rank)
    ((model(x) - y) ** 2).mean().div(2).backward()
    frozen = model.layers[0].up.weight
    return {"frozen_grad": frozen.grad is None, "frozen_rg": frozen.requires_grad,
            "grads": {n: _full(p.grad).clone() for n, p in model.named_parameters() if p.grad is not None},
            "reduced": ctl.stats()["bytes_reduced"]}


def test_symm_fsdp_frozen_weight():
    """A frozen linear keeps no gradient and moves no reduce-scatter traffic; the input gradient
    still flows through it to the layers below."""
    got = run_ranks(_frozen, 2)
    assert got["frozen_grad"] and not got["frozen_rg"]
    ref = Net()
    ref.layers[0].up.weight.requires_grad_(False)
    xs, ys = zip(*[_data(0, r) for r in range(2)])
    ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    names = {n for n, p in ref.named_parameters() if p.grad is not None}
    assert set(got["grads"]) == names
    for n, p in ref.named_parameters():
        if p.grad is not None:
            assert rel_err(got["grads"][n], p.grad) < 1e-5, n
    shard = ((H // 2) * D + (D // 2) * H) * 4  # one up and one down weight: the other rank's rows
    assert got["reduced"] == 2 * shard - (H // 2) * D * 4


def _pure_replication(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    mesh = init_device_mesh("cpu", (2, 1), mesh_dim_names=("replicate", "shard"))
    model = Net()
    ctl = apply_symm_fsdp(model, mesh=mesh)
    assert ctl.world == 1 and ctl.replicas == 2
    for mb in range(2):
        model.set_requires_gradient_sync(mb == 1)
        x, y = _data(mb, rank)
        ((model(x) - y) ** 2).mean().div(2).backward()
    return {n: _full(p.grad).clone() for n, p in model.named_parameters()}


def test_symm_fsdp_replicas_of_one_shard():
    """A (2, 1) mesh: every rank holds whole weights and only the replica average moves
    gradients; the result equals one process on the union of the data."""
    got = run_ranks(_pure_replication, 2)
    ref = Net()
    for mb in range(2):
        xs, ys = zip(*[_data(mb, r) for r in range(2)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().div(2).backward()
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.grad) < 1e-5, n


def _hdsp_on_symm(rank, world, steps):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import HDSPMuonOptimizer
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("replicate", "shard"))
    model = Net()
    ctl = apply_symm_fsdp(model, mesh=mesh)
    opt = HDSPMuonOptimizer(model, lr=0.02)
    assert opt.device_mesh is not None and opt.device_mesh.ndim == 2
    ctl.attach_optimizer(opt)
    for s in range(steps):
        x, y = _data(20 + s, rank)
        ((model(x) - y) ** 2).mean().backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
    return {n: _full(p.detach()).clone() for n, p in model.named_parameters()}


def test_hdsp_optimizer_on_fused_fsdp_hsdp():
    """HDSPMuonOptimizer finds the 2-D mesh of the fused-FSDP parameters and exchanges inside the
    shard groups: training equals one process on the union of the data."""
    from my_muon_fsdp2_b200 import HDSPMuonOptimizer

    steps = 2
    got = run_ranks(_hdsp_on_symm, 4, steps)
    ref = Net()
    opt = HDSPMuonOptimizer(ref, lr=0.02)
    for s in range(steps):
        xs, ys = zip(*[_data(20 + s, r) for r in range(4)])
        ((ref(torch.cat(xs)) - torch.cat(ys)) ** 2).mean().backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
    for n, p in ref.named_parameters():
        assert rel_err(got[n], p.detach()) < 1e-4, n


def _memory(rank, world):
    from my_muon_fsdp2_b200.parallel.symm_fsdp import apply_symm_fsdp

    model = Net()
    ctl = apply_symm_fsdp(model)
    before = ctl.memory_bytes()
    x, y = _data(0, rank)
    model.set_requires_gradient_sync(False)
    ((model(x) - y) ** 2).mean().backward()
    return before, ctl.memory_bytes()


def test_symm_fsdp_memory_report():
    before, after = run_ranks(_memory, 2)
    weights = 2 * (H * D + D * H) * 4  # two blocks of up + down, fp32
    assert before == {"shards": weights // 2, "full_weights": 0, "grad_accumulators": 0, "rs_slots": 0}
    # after a no-sync micro-batch: every weight gathered once and an unsharded accumulator each
    assert after["full_weights"] == weights and after["grad_accumulators"] == weights
