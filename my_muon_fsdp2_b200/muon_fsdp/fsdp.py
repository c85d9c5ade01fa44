"""``muon_fsdp.fsdp``: FSDP2 Muon optimizer and DTensor / FSDP module helpers (the reference's public names of src/muon_fsdp/fsdp.py:29-586)."""
from ..optim.fsdp_muon import FSDPMuonOptimizer, create_fsdp_muon_optimizer
from ..parallel.dtensor import get_dtensor_full_tensor, get_dtensor_local_tensor, is_dtensor
from ..parallel.fsdp_utils import collect_fsdp_modules, has_fsdp_modules

__all__ = ["FSDPMuonOptimizer", "create_fsdp_muon_optimizer", "is_dtensor", "get_dtensor_local_tensor",
           "get_dtensor_full_tensor", "collect_fsdp_modules", "has_fsdp_modules"]
