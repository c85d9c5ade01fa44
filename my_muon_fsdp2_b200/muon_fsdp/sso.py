"""``muon_fsdp.sso``: Spectral-Sphere optimizer."""
from ..optim.sso import SpectralSphereOptimizer

__all__ = ["SpectralSphereOptimizer"]
