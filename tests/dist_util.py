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


def run_ranks_some_die(fn, world, *args, timeout_s=120.0, attempts=3):
    """Like :func:`run_ranks`, but a rank may end its own process (a killed rank): returns rank 0's
    value and every rank's exit code (negative = the signal that ended it).  Rank 0 must survive;
    a run whose rank 0 failed (e.g. its rendezvous port was taken by a parallel test) is retried."""
    for attempt in range(attempts):
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "result.pt")
            ctx = mp.start_processes(_entry, args=(world, free_port(), fn, path, args), nprocs=world, join=False,
                                     start_method="spawn")
            for p in ctx.processes:
                p.join(timeout_s)
            codes = []
            for p in ctx.processes:
                if p.is_alive():  # a hung rank: end this test's own child, by its PID
                    p.kill()
                    p.join(5)
                codes.append(p.exitcode)
            if codes[0] != 0 and attempt + 1 < attempts:
                continue
            return (torch.load(path, weights_only=False) if os.path.exists(path) else None), codes
