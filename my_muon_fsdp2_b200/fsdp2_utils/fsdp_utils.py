"""``fsdp2_utils.fsdp_utils`` (the reference's public names of src/fsdp2_utils/fsdp_utils.py:19-119)."""
from ..parallel.fsdp_utils import (  # noqa: F401
    HAS_FSDP2,
    apply_local_updates,
    collect_fsdp_modules,
    get_local_grads,
    get_local_params,
    get_model_params_with_grad,
    has_fsdp_modules,
    is_fsdp_module,
    unshard_model,
    unshard_modules,
)
