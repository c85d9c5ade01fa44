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
    """Run fn(rank, world, *args) on `world` gloo ranks; return rank 0's return value.  A start-up
    that lost its rendezvous port to another process (tests run in parallel) is retried on a new
    port; any other failure propagates."""
    for attempt in range(3):
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "result.pt")
            try:
                mp.spawn(_entry, args=(world, free_port(), fn, path, args), nprocs=world, join=True)
            except mp.ProcessRaisedException as e:
                msg = str(e).lower()
                if attempt < 2 and ("address already in use" in msg or "eaddrinuse" in msg):
                    continue
                raise
            return torch.load(path, weights_only=False)
