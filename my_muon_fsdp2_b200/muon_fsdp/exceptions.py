"""``muon_fsdp.exceptions``: the optimizer exceptions of the reference's API guide
(docs/api.md:404-417), absent from its source tree."""
from ..optim.errors import InvalidParameterError, OptimizerError, SparseGradientError

__all__ = ["OptimizerError", "InvalidParameterError", "SparseGradientError"]
