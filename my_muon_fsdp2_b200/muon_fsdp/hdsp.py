"""``muon_fsdp.hdsp``: HSDP Muon optimizer and 2-D mesh helpers (the reference's public names of src/muon_fsdp/hdsp.py:49-486)."""
from ..optim.hdsp import HDSPMuonOptimizer, HSDPConfig
from ..parallel.dtensor import is_dtensor
from ..parallel.mesh import create_device_mesh_2d, gather_grads_group, get_hsdp_groups

__all__ = ["HDSPMuonOptimizer", "HSDPConfig", "create_device_mesh_2d", "get_hsdp_groups", "gather_grads_group",
           "is_dtensor"]
