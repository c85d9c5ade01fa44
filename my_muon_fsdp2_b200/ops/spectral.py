"""Spectral operations for the Spectral-Sphere optimizer.

Parity with ``src/muon_fsdp/spectral.py`` (power_iteration, compute_spectral_norm,
bisect_spectral_radius, compute_target_radius, apply_spectral_retraction) and with the symmetric
eigen-power iteration of ``src/fsdp2_utils/numerical.py:59-106``.

CUDA inputs use the device-resident power iteration kernel (GEMV + in-kernel normalisation);
sigma stays on the device unless the caller asks for a Python float.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn.functional as F


def _check2d(t: torch.Tensor) -> None:
    if t.dim() < 2:
        raise ValueError(f"Input tensor must have at least 2 dimensions, got {t.dim()}")


@torch.no_grad()
def power_iteration(tensor: torch.Tensor, num_iterations: int = 10, eps: float = 1e-7
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Leading singular triplet ``(sigma, u (m,1), v (n,1))`` with ``sigma = u^T W v``."""
    _check2d(tensor)
    w = tensor.reshape(tensor.shape[0], -1)
    m, n = w.shape
    if w.is_cuda:
        from .._ext import ext

        wc = w.contiguous()
        if wc.dtype not in (torch.float32, torch.bfloat16):
            wc = wc.float()
        v = torch.randn(n, device=w.device, dtype=torch.float32)
        u = torch.empty(m, device=w.device, dtype=torch.float32)
        sigma = torch.empty((), device=w.device, dtype=torch.float32)
        work = torch.empty(max(m, n) + 1, device=w.device, dtype=torch.float32)
        ext().power_iteration(wc, u, v, sigma, num_iterations, eps, work)
        return sigma, u.view(m, 1), v.view(n, 1)
    w = w.to(torch.float32)
    v = F.normalize(torch.randn(n, 1, dtype=torch.float32), dim=0, eps=eps)
    u = torch.zeros(m, 1)
    for _ in range(num_iterations):
        u = F.normalize(w @ v, dim=0, eps=eps)
        v = F.normalize(w.T @ u, dim=0, eps=eps)
    sigma = (u.T @ w @ v).squeeze()
    return sigma, u, v


def compute_spectral_norm(tensor: torch.Tensor, num_iterations: int = 10) -> float:
    """Largest singular value as a Python float (one device sync on CUDA)."""
    _check2d(tensor)
    sigma, _, _ = power_iteration(tensor, num_iterations=num_iterations)
    return float(sigma.item())


@torch.no_grad()
def bisect_spectral_radius(target_radius: float, matrix_dim: Tuple[int, int], max_iterations: int = 100,
                           tolerance: float = 1e-6) -> float:
    """Bisection for the Lagrange multiplier of the spectral-sphere constraint.

    The reference solves a *proxy* objective ``f(lam) = lam / sqrt(max(m, n)) - 0.1 R`` on the
    bracket ``[-R sqrt(max(m,n)), R sqrt(max(m,n))]`` (spectral.py:141-189) rather than the msign
    equation of the SSO paper; the same objective is kept here so that results agree.
    """
    if target_radius <= 0:
        raise ValueError(f"target_radius must be positive, got {target_radius}")
    m, n = matrix_dim
    scale = math.sqrt(max(m, n))
    lo, hi = -target_radius * scale, target_radius * scale

    def f(lam: float) -> float:
        return lam / scale - 0.1 * target_radius

    flo, fhi = f(lo), f(hi)
    if flo * fhi > 0:
        return 0.0
    for _ in range(max_iterations):
        mid = 0.5 * (lo + hi)
        fm = f(mid)
        if abs(fm) < tolerance:
            return mid
        if fm * flo < 0:
            hi, fhi = mid, fm
        else:
            lo, flo = mid, fm
    return 0.5 * (lo + hi)


@torch.no_grad()
def compute_target_radius(shape, radius_mode: str = "spectral_mup", radius_scaler: float = 1.0) -> float:
    """``spectral_mup``: R = s * sqrt(n_out / n_in); ``identity``: R = s."""
    if radius_mode == "spectral_mup":
        return radius_scaler * math.sqrt(shape[0] / shape[1])
    if radius_mode == "identity":
        return radius_scaler * 1.0
    raise ValueError(f"Invalid radius_mode: {radius_mode}. Must be one of: 'spectral_mup', 'identity'")


def retraction_scale(current_sigma, target_radius: float, mode: str = "hard", eps: float = 1e-8):
    """Multiplier that retracts W onto the sphere (float or device tensor, no host sync)."""
    if mode not in ("hard", "dynamic"):
        raise ValueError(f"Invalid retraction mode: {mode}. Must be 'hard' or 'dynamic'")
    if isinstance(current_sigma, torch.Tensor):
        s = current_sigma.float()
        if mode == "hard":
            far = (s - target_radius).abs() > eps
            return torch.where(far, target_radius / (s.clamp_min(0.0) + eps), torch.ones_like(s))
        return torch.where(s > target_radius, torch.full_like(s, 0.95), torch.full_like(s, 1.05))
    if mode == "hard":
        if abs(current_sigma - target_radius) > eps:
            return target_radius / (max(current_sigma, 0.0) + eps)
        return 1.0
    return 0.95 if current_sigma > target_radius else 1.05


@torch.no_grad()
def apply_spectral_retraction(weight: torch.Tensor, current_sigma, target_radius: float, mode: str = "hard",
                              eps: float = 1e-8) -> None:
    """In place: ``hard`` W *= R/(sigma+eps) when |sigma-R| > eps; ``dynamic`` W *= 1 -/+ 0.05."""
    scale = retraction_scale(current_sigma, target_radius, mode, eps)
    weight.mul_(scale)


# ---- fsdp2_utils.numerical variants (symmetric eigen power iteration) ----------------------
@torch.no_grad()
def power_iteration_symmetric(A: torch.Tensor, num_iterations: int = 100, tol: float = 1e-6):
    """Dominant eigenpair of a symmetric matrix: ``(float eigenvalue, v)``, early exit at ``tol``."""
    n = A.size(0)
    v = torch.randn(n, device=A.device, dtype=A.dtype)
    v = v / v.norm()
    for _ in range(num_iterations):
        w = A @ v
        w = w / w.norm()
        done = (v - w).norm() < tol
        v = w
        if bool(done):
            break
    return float((v @ A @ v).item()), v


@torch.no_grad()
def compute_spectral_norm_gram(A: torch.Tensor, num_iterations: int = 100) -> torch.Tensor:
    """sqrt(lambda_max) of the smaller Gram matrix (A^T A or A A^T), as a tensor."""
    if A.dim() == 2:
        m, n = A.shape
        B = A.T @ A if m >= n else A @ A.T
        lam, _ = power_iteration_symmetric(B, num_iterations)
        return torch.sqrt(torch.tensor(lam, device=A.device, dtype=A.dtype))
    return torch.linalg.norm(A, 2)
