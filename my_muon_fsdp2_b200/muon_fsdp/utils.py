"""``muon_fsdp.utils``: Newton–Schulz (see :mod:`my_muon_fsdp2_b200.ops.newton_schulz`) (the reference's public names of src/muon_fsdp/utils.py:12-106)."""
from ..ops.newton_schulz import NS_COEFFICIENTS, zeropower_via_newtonschulz5

__all__ = ["zeropower_via_newtonschulz5", "NS_COEFFICIENTS"]
