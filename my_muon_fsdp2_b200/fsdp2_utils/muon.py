"""``fsdp2_utils.muon``."""
from ..optim.fsdp2_muon import MuonOptimizer  # noqa: F401
