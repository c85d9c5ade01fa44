"""``muon_fsdp.distributed``: collective primitives (the reference's public names of src/muon_fsdp/distributed.py:13-170)."""
from ..parallel.comm import all_gather_grads, get_rank, get_world_size, is_available, scatter_updates

__all__ = ["is_available", "get_world_size", "get_rank", "all_gather_grads", "scatter_updates"]
