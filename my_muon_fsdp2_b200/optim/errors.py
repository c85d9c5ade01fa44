"""Optimizer exceptions documented in the reference's API guide (docs/api.md:404-417:
``muon_fsdp.exceptions`` with ``OptimizerError``, ``SparseGradientError`` and
``InvalidParameterError``), which its source tree does not ship.  They subclass the built-in
errors the optimizers have always raised (``ValueError`` for a bad hyperparameter,
``RuntimeError`` for a sparse gradient), so code that catches those keeps working."""


class OptimizerError(Exception):
    """Base class of the optimizer errors of this library."""


class InvalidParameterError(OptimizerError, ValueError):
    """A hyperparameter outside its valid range (learning rate, momentum, weight decay, ...)."""


class SparseGradientError(OptimizerError, RuntimeError):
    """A sparse gradient reached an optimizer that needs dense ones."""


__all__ = ["OptimizerError", "InvalidParameterError", "SparseGradientError"]
