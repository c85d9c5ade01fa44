"""my_muon_fsdp2_b200 — a Blackwell-native (sm_100a) FSDP2 + Muon training library.

The top level re-exports the ``muon_fsdp`` API (optimizers, Newton–Schulz, spectral ops,
collective and DTensor helpers) plus the hybrid builder and the fused AdamW.  The
``fsdp2_utils`` API lives in :mod:`my_muon_fsdp2_b200.fsdp2_utils`.
"""
from .version import __version__
from .muon_fsdp import (
    FSDPMuonOptimizer,
    HDSPMuonOptimizer,
    HSDPConfig,
    MuonOptimizer,
    SpectralSphereOptimizer,
    all_gather_grads,
    apply_spectral_retraction,
    bisect_spectral_radius,
    collect_fsdp_modules,
    compute_spectral_norm,
    compute_target_radius,
    create_device_mesh_2d,
    create_fsdp_muon_optimizer,
    gather_grads_group,
    get_dtensor_full_tensor,
    get_dtensor_local_tensor,
    get_hsdp_groups,
    has_fsdp_modules,
    is_dtensor,
    power_iteration,
    scatter_updates,
    zeropower_via_newtonschulz5,
)
from .optim.adamw import FusedAdamW
from .optim.hybrid import HybridMuonAdamW, HybridMuonAdamWOptimizer, create_hybrid_optimizer, is_hidden_matrix

__all__ = [
    "MuonOptimizer", "zeropower_via_newtonschulz5", "all_gather_grads", "scatter_updates", "FSDPMuonOptimizer",
    "create_fsdp_muon_optimizer", "is_dtensor", "get_dtensor_local_tensor", "get_dtensor_full_tensor",
    "collect_fsdp_modules", "has_fsdp_modules", "SpectralSphereOptimizer", "compute_spectral_norm",
    "power_iteration", "compute_target_radius", "apply_spectral_retraction", "bisect_spectral_radius",
    "HDSPMuonOptimizer", "HSDPConfig", "create_device_mesh_2d", "gather_grads_group", "get_hsdp_groups",
    "HybridMuonAdamW", "HybridMuonAdamWOptimizer", "create_hybrid_optimizer", "is_hidden_matrix", "FusedAdamW",
    "__version__",
]
