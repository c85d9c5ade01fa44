"""``fsdp2_utils.numerical``: NS and the symmetric eigen-power iteration helpers.

``power_iteration(A, num_iterations=100, tol=1e-6)`` returns ``(float eigenvalue, v)`` for a
symmetric ``A`` and ``compute_spectral_norm(A, num_iterations=100)`` returns a tensor, as in
``src/fsdp2_utils/numerical.py:59-106``.
"""
from ..ops.newton_schulz import zeropower_via_newtonschulz5  # noqa: F401
from ..ops.spectral import compute_spectral_norm_gram as compute_spectral_norm  # noqa: F401
from ..ops.spectral import power_iteration_symmetric as power_iteration  # noqa: F401

__all__ = ["zeropower_via_newtonschulz5", "power_iteration", "compute_spectral_norm"]
