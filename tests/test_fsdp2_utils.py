"""The ``fsdp2_utils`` helper API: single-process fallbacks, DTensor helpers and FSDP2 module
helpers on 2 gloo ranks, the FSDP-compatible optimizer base class, and the command lines
(the reference's fsdp2_utils package, src/fsdp2_utils/{comm,dtensor,fsdp_utils,base,cli}.py)."""
import pytest
import torch
import torch.nn as nn

from tests.dist_util import run_ranks


class TestSingleProcessFallbacks:
    """Without a process group every collective helper is the identity (comm.py:18-267)."""

    def test_queries(self):
        from my_muon_fsdp2_b200 import fsdp2_utils as fu

        assert not fu.is_distributed()
        assert fu.get_world_size() == 1 and fu.get_rank() == 0 and fu.get_local_rank() == 0

    def test_collectives_are_identity(self):
        from my_muon_fsdp2_b200 import fsdp2_utils as fu

        t = torch.arange(6.0).view(3, 2)
        assert fu.all_gather([t])[0] is t
        assert fu.all_gather_grads([t])[0] is t
        assert fu.scatter([t])[0] is t
        assert fu.scatter_updates([t])[0] is t
        assert fu.all_reduce(t) is t and fu.all_reduce_sum(t) is t and fu.all_reduce_avg(t) is t
        assert fu.broadcast(t) is t
        fu.barrier()
        assert torch.equal(t, torch.arange(6.0).view(3, 2))

    def test_plain_tensor_helpers(self):
        from my_muon_fsdp2_b200 import fsdp2_utils as fu

        t = torch.randn(4, 3)
        assert not fu.is_dtensor(t) and fu.get_local_tensor(t) is t and fu.get_full_tensor(t) is t
        assert fu.get_shard_dim(t) is None
        info = fu.dtensor_meta_info(t)
        assert info == {"is_dtensor": False, "local_shape": t.shape, "global_shape": t.shape, "shard_dim": None,
                        "device_mesh_shape": None}
        assert fu.HAS_DTENSOR and fu.HAS_FSDP2


def _dtensor_helpers(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from my_muon_fsdp2_b200 import fsdp2_utils as fu
    from my_muon_fsdp2_b200.parallel.dtensor import create_dtensor, redistribute_dtensor

    torch.manual_seed(0)
    full = torch.randn(6, 4)
    mesh = init_device_mesh("cpu", (world,))
    d0 = create_dtensor(full, mesh, shard_dim=0)
    d1 = create_dtensor(full, shard_dim=1)  # default mesh over the world
    rep = redistribute_dtensor(d0, replicate=True)
    moved = redistribute_dtensor(d0, shard_dim=1)
    return {
        "local0": tuple(fu.get_local_tensor(d0).shape), "local1": tuple(fu.get_local_tensor(d1).shape),
        "dims": (fu.get_shard_dim(d0), fu.get_shard_dim(d1), fu.get_shard_dim(rep)),
        "meta": fu.dtensor_meta_info(d0),
        "full_ok": bool(torch.equal(fu.get_full_tensor(d0), full) and torch.equal(fu.get_full_tensor(d1), full)),
        "rep_ok": bool(torch.equal(fu.get_local_tensor(rep), full)),
        "moved": (fu.get_shard_dim(moved), tuple(fu.get_local_tensor(moved).shape)),
        "moved_ok": bool(torch.equal(fu.get_full_tensor(moved), full)),
    }


def test_dtensor_helpers_on_two_ranks():
    got = run_ranks(_dtensor_helpers, 2)
    assert got["local0"] == (3, 4) and got["local1"] == (6, 2)
    assert got["dims"] == (0, 1, None)
    m = got["meta"]
    assert m["is_dtensor"] and m["shard_dim"] == 0 and m["device_mesh_shape"] == (2,)
    assert tuple(m["local_shape"]) == (3, 4)
    assert got["full_ok"] and got["rep_ok"] and got["moved_ok"]
    assert got["moved"] == (1, (6, 2))


def _fsdp_helpers(rank, world):
    from torch.distributed.fsdp import fully_shard

    from my_muon_fsdp2_b200 import fsdp2_utils as fu

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(8, 16), nn.ReLU(), nn.Linear(16, 4))
    for m in (model[0], model[2]):
        fully_shard(m)
    fully_shard(model)
    out = {"is_root": fu.is_fsdp_module(model), "n_modules": len(fu.collect_fsdp_modules(model)),
           "has": fu.has_fsdp_modules(model), "plain_has": fu.has_fsdp_modules(nn.Linear(2, 2))}
    local = [tuple(t.shape) for t in fu.get_local_params(list(model.parameters()))]
    out["local_shapes"] = local
    x = torch.randn(5, 8)
    model(x).sum().backward()
    params = fu.get_model_params_with_grad(model)
    out["with_grad"] = len(params)
    grads = fu.get_local_grads(params)
    out["grad_shapes"] = [tuple(g.shape) for g in grads]
    before = [t.clone() for t in fu.get_local_params(params)]
    fu.apply_local_updates(params, [torch.ones_like(t) for t in before])
    after = fu.get_local_params(params)
    out["updated"] = all(torch.equal(a, b + 1) for a, b in zip(after, before))
    with fu.unshard_model(model):
        out["unsharded_shape"] = tuple(model[0].weight.shape)
    return out


def test_fsdp_module_helpers_on_two_ranks():
    got = run_ranks(_fsdp_helpers, 2)
    assert got["is_root"] and got["has"] and not got["plain_has"]
    assert got["n_modules"] == 3
    assert got["local_shapes"] == [(8, 8), (8,), (2, 16), (2,)]
    assert got["with_grad"] == 4 and got["grad_shapes"] == got["local_shapes"]
    assert got["updated"]
    assert got["unsharded_shape"] == (16, 8)


class TestOptimizerBase:
    """FSDPCompatibleOptimizer (base.py:32-238): accumulation gate, step_count in the state dict."""

    def _make(self, k):
        from my_muon_fsdp2_b200.fsdp2_utils import FSDPCompatibleOptimizer

        class Sgd(FSDPCompatibleOptimizer):
            calls = 0

            def _step_impl(self):
                type(self).calls += 1
                params = [p for g in self.param_groups for p in g["params"]]
                grads = self._gather_gradients(params)
                ups = [None if g is None else -0.1 * g for g in grads]
                self._apply_updates(params, self._scatter_updates(params, ups))

        model = nn.Linear(4, 2)
        return Sgd(model, gradient_accumulation_steps=k), model

    def test_accumulation_gate(self):
        opt, model = self._make(3)
        w0 = model.weight.detach().clone()
        for _ in range(5):
            model(torch.randn(2, 4)).sum().backward()
            opt.step()
        assert type(opt).calls == 1 and opt._step_count == 5
        assert not torch.equal(model.weight.detach(), w0)

    def test_state_dict_step_count_roundtrip(self):
        opt, model = self._make(1)
        model(torch.randn(2, 4)).sum().backward()
        opt.step()
        sd = opt.state_dict()
        assert sd["step_count"] == 1 and {"state", "param_groups"} <= set(sd)
        opt2, _ = self._make(1)
        opt2.load_state_dict(sd)
        assert opt2._step_count == 1

    def test_zero_grad_keeps_or_drops(self):
        opt, model = self._make(1)
        model(torch.randn(2, 4)).sum().backward()
        opt.zero_grad()
        assert model.weight.grad is not None and float(model.weight.grad.abs().sum()) == 0.0
        opt.zero_grad(set_to_none=True)
        assert model.weight.grad is None

    def test_validation(self):
        from my_muon_fsdp2_b200.fsdp2_utils import FSDPCompatibleOptimizer

        with pytest.raises(ValueError, match="gradient_accumulation_steps"):
            FSDPCompatibleOptimizer(nn.Linear(2, 2), gradient_accumulation_steps=0)
        frozen = nn.Linear(2, 2).requires_grad_(False)
        with pytest.raises(ValueError, match="empty parameter list"):
            FSDPCompatibleOptimizer(frozen)


class TestCommandLines:
    def test_muon_fsdp_info_and_check(self, capsys):
        from my_muon_fsdp2_b200.cli import muon_fsdp_main

        assert muon_fsdp_main(["info", "-v"]) == 0
        out = capsys.readouterr().out
        assert "muon-fsdp version" in out and "MuonOptimizer" in out
        assert muon_fsdp_main(["check", "--full"]) == 0
        out = capsys.readouterr().out
        assert "OK MuonOptimizer step" in out and "All checks passed!" in out

    def test_fsdp2_utils_info_and_version(self, capsys):
        from my_muon_fsdp2_b200.cli import fsdp2_utils_main
        from my_muon_fsdp2_b200.fsdp2_utils import __version__

        assert fsdp2_utils_main(["--info"]) == 0
        assert "FSDP2 utilities" in capsys.readouterr().out
        with pytest.raises(SystemExit) as e:
            fsdp2_utils_main(["--version"])
        assert e.value.code == 0
        assert __version__ in capsys.readouterr().out


def _gather_dtensor(rank, world):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import distribute_tensor
    from torch.distributed.tensor.placement_types import Shard

    from my_muon_fsdp2_b200 import all_gather_grads

    torch.manual_seed(0)
    full = torch.randn(6, 3)
    mesh = init_device_mesh("cpu", (world,))
    d = distribute_tensor(full, mesh, [Shard(0)])
    plain = torch.full((2, 2), float(rank))
    g_d, g_p = all_gather_grads([d, plain])
    return {"dtensor_full": bool(torch.equal(g_d, full)) and not hasattr(g_d, "to_local"),
            "plain": g_p}


def test_all_gather_grads_accepts_fsdp2_gradients():
    """FSDP2 gradients are DTensors: they gather to their full plain tensors (the reference's
    helper fails on them with a missing sharding strategy); plain tensors concatenate along dim 0."""
    got = run_ranks(_gather_dtensor, 2)
    assert got["dtensor_full"]
    assert torch.equal(got["plain"], torch.tensor([[0.0, 0.0], [0.0, 0.0], [1.0, 1.0], [1.0, 1.0]]))


def _list_collectives(rank, world):
    import torch.distributed as dist

    from my_muon_fsdp2_b200 import fsdp2_utils as fu

    a, b = torch.tensor([1.0 + rank]), torch.tensor([10.0 * (rank + 1)])
    out = {"sum": [t.clone() for t in fu.all_reduce_sum([a.clone(), b.clone()])],
           "avg": [t.clone() for t in fu.all_reduce_avg([a.clone(), b.clone()])],
           "max": fu.all_reduce([a.clone()], op=dist.ReduceOp.MAX)[0],
           "bcast": fu.broadcast([torch.tensor([float(rank)]), torch.tensor([rank + 5.0])], src_rank=1)}
    return out


def test_collectives_take_lists_like_the_reference():
    """fsdp2_utils.comm takes lists of tensors and ``src_rank`` (src/fsdp2_utils/comm.py:180-244)."""
    got = run_ranks(_list_collectives, 2)
    assert [float(t) for t in got["sum"]] == [3.0, 30.0]
    assert [float(t) for t in got["avg"]] == [1.5, 15.0]
    assert float(got["max"]) == 2.0
    assert [float(t) for t in got["bcast"]] == [1.0, 6.0]
