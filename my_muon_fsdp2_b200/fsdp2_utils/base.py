"""``fsdp2_utils.base``."""
from ..optim.base import FSDPCompatibleOptimizer  # noqa: F401
