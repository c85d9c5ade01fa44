"""CPU tests of the optimizers against restated reference math (tests/test_optimizer.py,
tests/test_sso.py, tests/test_hdsp.py of the reference, plus numeric oracles)."""
import copy
import io

import pytest
import torch
import torch.nn as nn

from my_muon_fsdp2_b200 import (
    FSDPMuonOptimizer,
    HDSPMuonOptimizer,
    HSDPConfig,
    HybridMuonAdamW,
    MuonOptimizer,
    SpectralSphereOptimizer,
    create_fsdp_muon_optimizer,
    create_hybrid_optimizer,
)
from my_muon_fsdp2_b200.fsdp2_utils import MuonOptimizer as ModelMuon
from tests.conftest import rel_err
from tests.oracle import muon_reference_step


def _model(seed=0):
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(32, 48), nn.GELU(), nn.Linear(48, 16))


def _loss(m, seed=1):
    torch.manual_seed(seed)
    dt = next(m.parameters()).dtype
    x, y = torch.randn(8, 32, dtype=dt), torch.randn(8, 16, dtype=dt)
    return ((m(x) - y) ** 2).mean()


class TestMuonOptimizer:
    def test_defaults(self):
        opt = MuonOptimizer(_model().parameters())
        g = opt.param_groups[0]
        assert (g["lr"], g["momentum"], g["weight_decay"], g["nesterov"], g["ns_steps"]) == (0.02, 0.95, 0.0, False, 5)

    @pytest.mark.parametrize("kw,msg", [({"lr": -0.01}, "Invalid learning rate"), ({"momentum": 1.5}, "Invalid momentum"),
                                        ({"weight_decay": -0.01}, "Invalid weight_decay"),
                                        ({"ns_steps": -1}, "Invalid ns_steps"),
                                        ({"nesterov": True, "momentum": 0.0}, "Nesterov momentum requires")])
    def test_validation(self, kw, msg):
        with pytest.raises(ValueError, match=msg):
            MuonOptimizer(_model().parameters(), **kw)

    @pytest.mark.parametrize("nesterov", [False, True])
    @pytest.mark.parametrize("wd", [0.0, 0.1])
    def test_matches_reference_math(self, nesterov, wd):
        m = _model().double()
        ref = copy.deepcopy(m)
        opt = MuonOptimizer(m.parameters(), lr=0.05, momentum=0.9, weight_decay=wd, nesterov=nesterov)
        bufs = [torch.zeros_like(p) for p in ref.parameters()]
        for step in range(3):
            opt.zero_grad()
            _loss(m, step).backward()
            opt.step()
            for p in ref.parameters():
                p.grad = None
            _loss(ref, step).backward()
            with torch.no_grad():
                muon_reference_step(list(ref.parameters()), [p.grad for p in ref.parameters()], bufs, 0.05, 0.9, wd,
                                    nesterov, 5)
        for p, q in zip(m.parameters(), ref.parameters()):
            assert rel_err(p, q) < 1e-9

    def test_sparse_grad_error(self):
        emb = nn.Embedding(10, 4, sparse=True)
        opt = MuonOptimizer(emb.parameters())
        emb(torch.tensor([1, 2])).sum().backward()
        with pytest.raises(RuntimeError, match="sparse gradients"):
            opt.step()

    def test_closure_and_state_roundtrip(self):
        m = _model()
        opt = MuonOptimizer(m.parameters())

        def closure():
            opt.zero_grad()
            loss = _loss(m)
            loss.backward()
            return loss

        assert opt.step(closure) is not None
        sd = opt.state_dict()
        assert all("momentum_buffer" in v for v in sd["state"].values())
        buf = io.BytesIO()
        torch.save(sd, buf)
        buf.seek(0)
        m2 = copy.deepcopy(m)
        opt2 = MuonOptimizer(m2.parameters())
        opt2.load_state_dict(torch.load(buf))
        for p, q in zip(m.parameters(), m2.parameters()):
            assert torch.equal(opt.state[p]["momentum_buffer"], opt2.state[q]["momentum_buffer"])

    def test_converges_on_small_problem(self):
        torch.manual_seed(0)
        lin = nn.Linear(16, 16, bias=False)
        target = torch.randn(16, 16)
        opt = MuonOptimizer(lin.parameters(), lr=0.02)
        x = torch.randn(64, 16)
        first = None
        for _ in range(100):
            opt.zero_grad()
            loss = ((lin(x) - x @ target.T) ** 2).mean()
            first = first if first is not None else loss.item()
            loss.backward()
            opt.step()
        assert loss.item() < 0.5 * first


class TestFSDPMuon:
    def test_defaults_and_state_layout(self):
        m = _model()
        opt = FSDPMuonOptimizer(m)
        g = opt.param_groups[0]
        for k, v in dict(lr=0.02, weight_decay=0.01, momentum=0.95, nesterov=True, ns_steps=5, ns_stepsize=1.0,
                         beta2=0.99, eps=1e-8).items():
            assert g[k] == v
        for p in m.parameters():
            assert set(opt.state[p]) == {"momentum_buffer", "second_moment", "accum_count"}
        sd = opt.state_dict()
        assert set(sd) == {"state", "param_groups", "step_count"}

    def test_empty_params(self):
        m = _model()
        for p in m.parameters():
            p.requires_grad_(False)
        with pytest.raises(ValueError, match="empty parameter list"):
            FSDPMuonOptimizer(m)

    def test_muon_rule_matches_oracle_with_stepsize(self):
        m = _model().double()
        ref = copy.deepcopy(m)
        opt = create_fsdp_muon_optimizer(m, lr=0.04, weight_decay=0.01, momentum=0.9, nesterov=True, ns_stepsize=0.5)
        bufs = [torch.zeros_like(p) for p in ref.parameters()]
        for step in range(2):
            opt.zero_grad()
            _loss(m, step).backward()
            opt.step()
            for p in ref.parameters():
                p.grad = None
            _loss(ref, step).backward()
            with torch.no_grad():
                # lr*ns_stepsize is the step; weight decay uses lr (1 - lr*wd)
                for p, b in zip(ref.parameters(), bufs):
                    b.lerp_(p.grad, 0.1)
                    u = p.grad + 0.9 * b
                    if p.dim() == 2:
                        from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference

                        u = newton_schulz_reference(u)
                    p.mul_(1 - 0.04 * 0.01)
                    p.add_(u, alpha=-0.04 * 0.5)
        for p, q in zip(m.parameters(), ref.parameters()):
            assert rel_err(p, q) < 1e-9

    def test_reference_rule_literal_update(self):
        m = _model().double()
        before = [p.detach().clone() for p in m.parameters()]
        opt = FSDPMuonOptimizer(m, update_rule="reference", ns_stepsize=0.3)
        _loss(m).backward()
        grads = [p.grad.clone() for p in m.parameters()]
        opt.step()
        from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference

        for p, b, g in zip(m.parameters(), before, grads):
            u = -0.3 * (newton_schulz_reference(g) if g.dim() == 2 else g)
            assert rel_err(p - b, u) < 1e-6

    def test_gradient_accumulation_gate(self):
        m = _model()
        opt = FSDPMuonOptimizer(m, gradient_accumulation_steps=2)
        before = [p.detach().clone() for p in m.parameters()]
        _loss(m).backward()
        opt.step()
        assert all(torch.equal(p, b) for p, b in zip(m.parameters(), before))
        opt.step()
        assert any(not torch.equal(p, b) for p, b in zip(m.parameters(), before))
        assert opt.state_dict()["step_count"] == 2

    def test_zero_grad_keeps_tensors(self):
        m = _model()
        opt = FSDPMuonOptimizer(m)
        _loss(m).backward()
        opt.zero_grad()
        assert all(p.grad is not None and p.grad.abs().sum() == 0 for p in m.parameters())

    def test_unshard_params_noop_without_fsdp(self):
        opt = FSDPMuonOptimizer(_model())
        with opt.unshard_params():
            pass


class TestModelFirstMuon:
    def test_coupled_weight_decay_and_persistent_momentum(self):
        m = _model().double()
        opt = ModelMuon(m, lr=0.05, momentum=0.9, weight_decay=0.1, nesterov=True)
        ref = copy.deepcopy(m)
        bufs = [torch.zeros_like(p) for p in ref.parameters()]
        from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference

        for step in range(2):
            opt.zero_grad()
            _loss(m, step).backward()
            opt.step()
            for p in ref.parameters():
                p.grad = None
            _loss(ref, step).backward()
            with torch.no_grad():
                for p, b in zip(ref.parameters(), bufs):
                    g = p.grad + 0.1 * p
                    b.lerp_(g, 0.1)
                    u = g + 0.9 * b
                    if p.dim() == 2:
                        u = newton_schulz_reference(u)
                    p.add_(u, alpha=-0.05)
        for p, q in zip(m.parameters(), ref.parameters()):
            assert rel_err(p, q) < 1e-9
        assert all(opt.state[p]["momentum_buffer"].abs().sum() > 0 for p in m.parameters())
        assert opt.state_dict()["step_count"] == 2


class TestHybrid:
    def test_routes_and_counts(self):
        m = _model()
        h = create_hybrid_optimizer(m)
        st = h.statistics()
        assert st["muon_params"] == 2 and st["adamw_params"] == 2
        _loss(m).backward()
        h.step()
        assert all("momentum_buffer" in h.optimizer.state[p] for p in h.muon_params)
        assert all(h.optimizer.state[p]["step"] == 1 for p in h.adamw_params)

    def test_adamw_branch_matches_torch_adamw(self):
        torch.manual_seed(0)
        p1 = nn.Parameter(torch.randn(10, dtype=torch.float64))
        p2 = nn.Parameter(p1.detach().clone())
        h = HybridMuonAdamW([p1], adamw_lr=1e-2, adamw_weight_decay=0.05)
        t = torch.optim.AdamW([p2], lr=1e-2, weight_decay=0.05)
        for s in range(3):
            g = torch.randn(10, dtype=torch.float64)
            p1.grad, p2.grad = g.clone(), g.clone()
            h.step()
            t.step()
        assert rel_err(p1, p2) < 1e-12

    def test_reference_compat_reproduces_division_by_zero(self):
        p = nn.Parameter(torch.randn(4))
        h = HybridMuonAdamW([p], reference_compat=True)
        p.grad = torch.randn(4)
        with pytest.raises(ZeroDivisionError):
            h.step()


class TestSSO:
    def test_validation(self):
        ps = _model().parameters()
        with pytest.raises(ValueError, match="Invalid power_iteration_steps"):
            SpectralSphereOptimizer(ps, power_iteration_steps=0)
        with pytest.raises(ValueError, match="Invalid radius_mode"):
            SpectralSphereOptimizer(_model().parameters(), radius_mode="invalid")
        with pytest.raises(ValueError, match="Invalid retract_mode"):
            SpectralSphereOptimizer(_model().parameters(), retract_mode="invalid")

    def test_retracts_towards_radius(self):
        torch.manual_seed(0)
        lin = nn.Linear(64, 64, bias=False)
        with torch.no_grad():
            lin.weight.mul_(10)
        opt = SpectralSphereOptimizer(lin.parameters(), lr=1e-3, radius_mode="identity", power_iteration_steps=30)
        for _ in range(3):
            opt.zero_grad()
            lin(torch.randn(8, 64)).pow(2).mean().backward()
            opt.step()
        sig = torch.linalg.matrix_norm(lin.weight.detach(), 2).item()
        assert abs(sig - 1.0) < 0.2
        info = opt.get_spectral_norms()[id(lin.weight)]
        assert {"current_sigma", "target_radius", "initial_sigma"} <= set(info)


class TestHDSP:
    def test_step_runs_single_process(self):
        m = _model().double()
        opt = HDSPMuonOptimizer(m, lr=0.01)
        before = [p.detach().clone() for p in m.parameters()]
        _loss(m).backward()
        opt.step()
        assert all(not torch.equal(p, b) for p, b in zip(m.parameters(), before))
        sd = opt.state_dict()
        assert set(sd) == {"step_count", "param_groups"} and sd["param_groups"][0]["params"] == []
        assert len(opt.param_groups[0]["params"]) == 4  # not mutated

    def test_hsdp_scale_math(self):
        from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference

        torch.manual_seed(0)
        w = nn.Parameter(torch.randn(8, 32, dtype=torch.float64))
        opt = HDSPMuonOptimizer(nn.Module(), params=[w], lr=0.1, weight_decay=0.0, momentum=0.9, nesterov=False)
        w0 = w.detach().clone()
        w.grad = torch.randn(8, 32, dtype=torch.float64)
        g = w.grad.clone()
        opt.step()
        u = newton_schulz_reference(0.1 * g)  # EMA buffer after one step = (1-mu) g
        assert rel_err(w - w0, -0.1 * 2.0 * u) < 1e-9  # sqrt(32/8) = 2

    def test_config(self):
        c = HSDPConfig(dp_size=2, fsdp_size=4)
        assert c.to_dict()["fsdp_size"] == 4
        assert c.create_device_mesh() is None  # no process group


def test_workload_registry_and_cli():
    from my_muon_fsdp2_b200.cli import muon_fsdp_main
    from my_muon_fsdp2_b200.configs import WORKLOADS, describe

    assert set(WORKLOADS) == {"mlp_gloo", "encoder", "gpt2_small", "llama3_8b", "muon_sweep"}
    assert all("command" in v for v in describe().values())
    assert muon_fsdp_main(["configs"]) == 0


def test_nvtx_ranges_are_noops_when_disabled():
    from my_muon_fsdp2_b200.utils import tracing

    tracing.enable(False)
    with tracing.nvtx_range("x"):
        pass
    assert not tracing.enabled()


def test_documented_exceptions():
    """muon_fsdp.exceptions (the reference's API guide) with the built-in bases kept."""
    import torch.nn as nn

    from my_muon_fsdp2_b200 import MuonOptimizer, SpectralSphereOptimizer
    from my_muon_fsdp2_b200.muon_fsdp.exceptions import InvalidParameterError, OptimizerError, SparseGradientError

    assert issubclass(InvalidParameterError, (OptimizerError, ValueError))
    assert issubclass(SparseGradientError, (OptimizerError, RuntimeError))
    with pytest.raises(InvalidParameterError):
        MuonOptimizer(nn.Linear(2, 2).parameters(), lr=-1.0)
    with pytest.raises(InvalidParameterError):
        SpectralSphereOptimizer(nn.Linear(2, 2).parameters(), radius_mode="nope")
    emb = nn.Embedding(10, 4, sparse=True)
    opt = MuonOptimizer(emb.parameters(), lr=0.01)
    emb(torch.tensor([1, 2])).sum().backward()
    with pytest.raises(SparseGradientError):
        opt.step()


def test_grad_scaler_drives_muon_like_a_plain_step():
    """torch.amp.GradScaler (the reference's mixed-precision recipe) unscales the gradients
    before MuonOptimizer.step: the update equals the one without scaling."""
    import copy

    import torch.nn as nn

    from my_muon_fsdp2_b200 import MuonOptimizer

    torch.manual_seed(0)
    a = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 8))
    b = copy.deepcopy(a)
    x, y = torch.randn(4, 16), torch.randn(4, 8)
    oa = MuonOptimizer(a.parameters(), lr=0.02, weight_decay=0.01)
    ob = MuonOptimizer(b.parameters(), lr=0.02, weight_decay=0.01)
    scaler = torch.amp.GradScaler("cpu", init_scale=1024.0)
    scaler.scale(((a(x) - y) ** 2).mean()).backward()
    scaler.step(oa)
    scaler.update()
    ((b(x) - y) ** 2).mean().backward()
    ob.step()
    for p, q in zip(a.parameters(), b.parameters()):
        assert torch.allclose(p, q, rtol=1e-5, atol=1e-6)
