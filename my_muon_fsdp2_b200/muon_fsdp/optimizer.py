"""``muon_fsdp.optimizer``: single-entry Muon optimizer."""
from ..optim.muon import MuonOptimizer

__all__ = ["MuonOptimizer"]
