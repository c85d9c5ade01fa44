"""``fsdp2_utils.comm`` (the reference's public names of src/fsdp2_utils/comm.py:18-267)."""
from ..parallel.comm import (  # noqa: F401
    all_gather,
    all_gather_grads,
    all_reduce,
    all_reduce_avg,
    all_reduce_sum,
    barrier,
    broadcast,
    get_local_rank,
    get_rank,
    get_world_size,
    is_distributed,
    scatter,
    scatter_updates,
)
