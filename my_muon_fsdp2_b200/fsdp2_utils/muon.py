"""``fsdp2_utils.muon`` (the reference's public names of src/fsdp2_utils/muon.py:14-144)."""
from ..optim.fsdp2_muon import MuonOptimizer  # noqa: F401
