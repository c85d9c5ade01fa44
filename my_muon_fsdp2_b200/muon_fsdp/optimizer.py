"""``muon_fsdp.optimizer``: single-entry Muon optimizer (the reference's public names of src/muon_fsdp/optimizer.py:15-190)."""
from ..optim.muon import MuonOptimizer

__all__ = ["MuonOptimizer"]
