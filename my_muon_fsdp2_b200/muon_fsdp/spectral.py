"""``muon_fsdp.spectral``: spectral operations for SSO (the reference's public names of src/muon_fsdp/spectral.py:18-282)."""
from ..ops.spectral import (
    apply_spectral_retraction,
    bisect_spectral_radius,
    compute_spectral_norm,
    compute_target_radius,
    power_iteration,
)

__all__ = ["compute_spectral_norm", "power_iteration", "bisect_spectral_radius", "compute_target_radius",
           "apply_spectral_retraction"]
