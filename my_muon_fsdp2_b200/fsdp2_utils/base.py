"""``fsdp2_utils.base`` (the reference's public names of src/fsdp2_utils/base.py:32-238)."""
from ..optim.base import FSDPCompatibleOptimizer  # noqa: F401
