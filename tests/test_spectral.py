"""Spectral operations and the Spectral-Sphere optimizer on CPU, against torch.linalg (the
reference's tests/test_sso.py cover the same behaviours: power iteration within 10 % of the
SVD, unit singular vectors, a finite bisection root, the target radius rules, hard / dynamic
retraction, the SSO state and its spectral-norm report)."""
import math

import pytest
import torch

from my_muon_fsdp2_b200 import (
    SpectralSphereOptimizer,
    apply_spectral_retraction,
    bisect_spectral_radius,
    compute_spectral_norm,
    compute_target_radius,
    power_iteration,
)
from my_muon_fsdp2_b200.fsdp2_utils import numerical


def _sigma_max(w):
    return float(torch.linalg.svdvals(w.double())[0])


class TestPowerIteration:
    @pytest.mark.parametrize("shape", [(64, 64), (128, 32), (32, 128), (256, 256)])
    def test_close_to_svd(self, shape):
        torch.manual_seed(0)
        w = torch.randn(*shape)
        sigma, u, v = power_iteration(w, num_iterations=50)
        assert abs(float(sigma) - _sigma_max(w)) / _sigma_max(w) < 0.1

    def test_triplet_shapes_and_unit_vectors(self):
        torch.manual_seed(1)
        w = torch.randn(48, 20)
        sigma, u, v = power_iteration(w, num_iterations=30)
        assert u.shape == (48, 1) and v.shape == (20, 1) and sigma.dim() == 0
        assert abs(float(u.norm()) - 1) < 1e-5 and abs(float(v.norm()) - 1) < 1e-5
        # sigma is u^T W v
        assert abs(float(sigma) - float(u.T @ w @ v)) < 1e-4

    def test_rank_one_is_exact(self):
        a, b = torch.randn(30, 1), torch.randn(1, 40)
        w = a @ b
        assert abs(compute_spectral_norm(w, num_iterations=5) - float(a.norm() * b.norm())) < 1e-3 * float(
            a.norm() * b.norm())

    def test_compute_spectral_norm_is_float(self):
        w = torch.randn(16, 16)
        s = compute_spectral_norm(w, num_iterations=40)
        assert isinstance(s, float) and abs(s - _sigma_max(w)) / _sigma_max(w) < 0.1

    def test_rejects_vectors(self):
        with pytest.raises(ValueError, match="at least 2 dimensions"):
            power_iteration(torch.randn(5))
        with pytest.raises(ValueError, match="at least 2 dimensions"):
            compute_spectral_norm(torch.randn(5))


class TestSymmetricPowerIteration:
    def test_dominant_eigenvalue(self):
        torch.manual_seed(2)
        a = torch.randn(40, 40, dtype=torch.float64)
        s = a @ a.T  # symmetric positive semi-definite
        lam, v = numerical.power_iteration(s, num_iterations=500, tol=1e-10)
        assert isinstance(lam, float)
        assert abs(lam - float(torch.linalg.eigvalsh(s)[-1])) / lam < 1e-6
        assert abs(float(v.norm()) - 1) < 1e-9

    def test_spectral_norm_from_the_smaller_gram(self):
        torch.manual_seed(3)
        for shape in [(50, 20), (20, 50)]:
            a = torch.randn(*shape, dtype=torch.float64)
            got = float(numerical.compute_spectral_norm(a, num_iterations=500))
            assert abs(got - _sigma_max(a)) / _sigma_max(a) < 1e-6


class TestRadiusAndBisection:
    def test_target_radius_rules(self):
        assert compute_target_radius((512, 128)) == pytest.approx(2.0)
        assert compute_target_radius((128, 512), radius_scaler=3.0) == pytest.approx(1.5)
        assert compute_target_radius((7, 3), radius_mode="identity", radius_scaler=0.5) == 0.5
        with pytest.raises(ValueError, match="radius_mode"):
            compute_target_radius((4, 4), radius_mode="nope")

    def test_bisection_root_of_the_proxy_objective(self):
        # the reference's objective f(lam) = lam / sqrt(max(m, n)) - 0.1 R has its root at
        # lam = 0.1 R sqrt(max(m, n))
        lam = bisect_spectral_radius(2.0, (64, 256), tolerance=1e-9)
        assert math.isfinite(lam)
        assert lam == pytest.approx(0.1 * 2.0 * 16.0, rel=1e-6)

    def test_bisection_rejects_nonpositive_radius(self):
        with pytest.raises(ValueError):
            bisect_spectral_radius(0.0, (4, 4))


class TestRetraction:
    def test_hard_lands_on_the_radius(self):
        torch.manual_seed(4)
        w = torch.randn(64, 32)
        s = _sigma_max(w)
        apply_spectral_retraction(w, s, 1.5, mode="hard")
        assert _sigma_max(w) == pytest.approx(1.5, rel=1e-5)

    def test_hard_leaves_a_weight_on_the_sphere(self):
        w = torch.randn(8, 8)
        before = w.clone()
        apply_spectral_retraction(w, 2.0, 2.0, mode="hard")
        assert torch.equal(w, before)

    def test_dynamic_steps(self):
        w = torch.ones(4, 4)
        apply_spectral_retraction(w, 3.0, 1.0, mode="dynamic")
        assert torch.allclose(w, torch.full((4, 4), 0.95))
        w = torch.ones(4, 4)
        apply_spectral_retraction(w, 0.5, 1.0, mode="dynamic")
        assert torch.allclose(w, torch.full((4, 4), 1.05))

    def test_tensor_sigma_matches_float_sigma(self):
        w1, w2 = torch.randn(6, 6), None
        w2 = w1.clone()
        apply_spectral_retraction(w1, 3.0, 1.2, mode="hard")
        apply_spectral_retraction(w2, torch.tensor(3.0), 1.2, mode="hard")
        assert torch.allclose(w1, w2)

    def test_invalid_mode(self):
        with pytest.raises(ValueError, match="retraction mode"):
            apply_spectral_retraction(torch.ones(2, 2), 1.0, 1.0, mode="soft")


class TestSpectralSphereOptimizer:
    def _model(self):
        torch.manual_seed(5)
        return torch.nn.Sequential(torch.nn.Linear(32, 64), torch.nn.ReLU(), torch.nn.Linear(64, 16))

    def test_state_keys_and_report(self):
        model = self._model()
        opt = SpectralSphereOptimizer(model.parameters(), lr=0.01, power_iteration_steps=20)
        x = torch.randn(8, 32)
        model(x).pow(2).mean().backward()
        opt.step()
        w = model[0].weight
        st = opt.state[w]
        assert {"momentum_buffer", "initial_sigma", "current_sigma", "target_radius"} <= set(st)
        assert st["target_radius"] == pytest.approx(math.sqrt(64 / 32))
        assert "initial_sigma" not in opt.state[model[0].bias]  # 1-D: no spectral state
        report = opt.get_spectral_norms()
        assert set(report) == {id(model[0].weight), id(model[2].weight)}
        assert report[id(w)]["target_radius"] == pytest.approx(math.sqrt(2.0))

    def test_weights_move_to_the_sphere(self):
        model = self._model()
        opt = SpectralSphereOptimizer(model.parameters(), lr=1e-4, power_iteration_steps=30, retract_mode="hard")
        for _ in range(3):
            opt.zero_grad()
            model(torch.randn(8, 32)).pow(2).mean().backward()
            opt.step()
        for lin in (model[0], model[2]):
            R = compute_target_radius(tuple(lin.weight.shape))
            assert abs(_sigma_max(lin.weight.detach()) - R) / R < 0.2

    def test_state_dict_roundtrip(self):
        model = self._model()
        opt = SpectralSphereOptimizer(model.parameters(), lr=0.01)
        model(torch.randn(8, 32)).pow(2).mean().backward()
        opt.step()
        sd = opt.state_dict()
        assert {"state", "param_groups"} <= set(sd)
        g = sd["param_groups"][0]
        for k in ("power_iteration_steps", "radius_mode", "radius_scaler", "retract_mode"):
            assert k in g
        opt2 = SpectralSphereOptimizer(model.parameters(), lr=0.01)
        opt2.load_state_dict(sd)
        for p in model.parameters():
            assert torch.equal(opt2.state[p]["momentum_buffer"], opt.state[p]["momentum_buffer"])
