"""``muon_fsdp`` API namespace (the reference package's public names, ``src/muon_fsdp/__init__.py:27-79``)."""
from ..version import __version__
from .distributed import all_gather_grads, scatter_updates
from .fsdp import (
    FSDPMuonOptimizer,
    collect_fsdp_modules,
    create_fsdp_muon_optimizer,
    get_dtensor_full_tensor,
    get_dtensor_local_tensor,
    has_fsdp_modules,
    is_dtensor,
)
from .hdsp import HDSPMuonOptimizer, HSDPConfig, create_device_mesh_2d, gather_grads_group, get_hsdp_groups
from .optimizer import MuonOptimizer
from .spectral import (
    apply_spectral_retraction,
    bisect_spectral_radius,
    compute_spectral_norm,
    compute_target_radius,
    power_iteration,
)
from .sso import SpectralSphereOptimizer
from .utils import zeropower_via_newtonschulz5

__all__ = [
    "MuonOptimizer", "zeropower_via_newtonschulz5", "all_gather_grads", "scatter_updates", "FSDPMuonOptimizer",
    "create_fsdp_muon_optimizer", "is_dtensor", "get_dtensor_local_tensor", "get_dtensor_full_tensor",
    "collect_fsdp_modules", "has_fsdp_modules", "SpectralSphereOptimizer", "compute_spectral_norm",
    "power_iteration", "compute_target_radius", "apply_spectral_retraction", "bisect_spectral_radius",
    "HDSPMuonOptimizer", "HSDPConfig", "create_device_mesh_2d", "gather_grads_group", "get_hsdp_groups",
    "__version__",
]
