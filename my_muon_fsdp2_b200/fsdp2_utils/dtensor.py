"""``fsdp2_utils.dtensor`` (the reference's public names of src/fsdp2_utils/dtensor.py:17-193)."""
from ..parallel.dtensor import (  # noqa: F401
    HAS_DTENSOR,
    create_dtensor,
    dtensor_meta_info,
    get_full_tensor,
    get_local_tensor,
    get_shard_dim,
    is_dtensor,
    redistribute_dtensor,
)
