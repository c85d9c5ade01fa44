"""``muon_fsdp.sso``: Spectral-Sphere optimizer (the reference's public names of src/muon_fsdp/sso.py:34-292)."""
from ..optim.sso import SpectralSphereOptimizer

__all__ = ["SpectralSphereOptimizer"]
