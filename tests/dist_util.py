"""Helpers for multi-process CPU (gloo) tests: spawn ranks, collect rank-0 results."""
import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import free_port


def _entry(rank, world, port, fn, result_path, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = fn(rank, world, *args)
        if rank == 0:
            torch.save(out, result_path)
    finally:
        dist.destroy_process_group()


def run_ranks(fn, world, *args):
    """Run fn(rank, world, *args) on `world` gloo ranks; return rank 0's return value."""
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "result.pt")
        mp.spawn(_entry, args=(world, free_port(), fn, path, args), nprocs=world, join=True)
        return torch.load(path, weights_only=False)
