"""Failure detection on CPU gloo ranks (host-side faults only): a rank that raises, a rank whose
process is killed, a rank that stops heart-beating, a delayed rank caught by a monitored
barrier, a corrupted replica."""
import datetime
import os
import signal
import time

import pytest
import torch
import torch.distributed as dist

from tests.dist_util import run_ranks, run_ranks_some_die

pytestmark = pytest.mark.distributed


def _heartbeat_dead_rank(rank, world):
    from my_muon_fsdp2_b200.parallel.fault import FaultInjector, Heartbeat, RankFailure

    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, interval_s=0.05).start()
    inj = FaultInjector(rank, hang_at=(1, 2, 2.0))
    detected = None
    for step in range(4):
        dist.barrier() if step < 2 else None
        if step == 2:
            try:
                inj.on_step(step, hb)  # rank 1 stops heart-beating and sleeps
                if rank == 0:
                    t0 = time.time()
                    while time.time() - t0 < 3.0:
                        try:
                            hb.check(limit_s=0.5)
                        except RankFailure as e:
                            detected = (e.ranks, round(time.time() - t0, 2))
                            break
                        time.sleep(0.05)
            finally:
                pass
            break
    hb.stop()
    return detected


def test_heartbeat_detects_hung_rank():
    ranks, t = run_ranks(_heartbeat_dead_rank, 2)
    assert ranks == [1] and t < 2.0


def _raising_rank(rank, world):
    from my_muon_fsdp2_b200.parallel.fault import FaultInjector, Heartbeat, RankFailure, guarded_barrier

    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, interval_s=0.05).start()
    inj = FaultInjector(rank, raise_at=(1, 1))
    out = None
    dist.barrier()  # both ranks start together, however late either process came up
    for step in range(3):
        try:
            inj.on_step(step, hb)
        except RuntimeError:
            hb.stop()  # the failed rank leaves between steps
            time.sleep(2.5)
            return None
        try:
            # step 0 is fault-free: a generous limit keeps a loaded machine from tripping it
            guarded_barrier(timeout_s=1.0 if step > 0 else 10.0, heartbeat=hb if step > 0 else None)
        except RankFailure as e:
            out = {"step": step, "ranks": e.ranks}
            break
    hb.stop()
    return out


def test_raising_rank_detected_before_next_collective():
    out = run_ranks(_raising_rank, 2)
    assert out is not None and out["step"] == 1 and out["ranks"] == [1]


def _killed_rank(rank, world):
    from my_muon_fsdp2_b200.parallel.fault import Heartbeat, RankFailure, guarded_barrier

    store = dist.distributed_c10d._get_default_store()  # served by rank 0's process
    hb = Heartbeat(store, rank, world, interval_s=0.05).start()
    dist.barrier()  # both ranks start together, however late either process came up
    out = None
    for step in range(3):
        if rank == 1 and step == 1:
            os.kill(os.getpid(), signal.SIGKILL)  # the process dies between steps
        try:
            guarded_barrier(timeout_s=1.0 if step > 0 else 10.0, heartbeat=hb if step > 0 else None)
        except RankFailure as e:
            out = {"step": step, "ranks": e.ranks}
            break
    hb.stop()
    return out


def test_killed_rank_detected_and_named():
    out, codes = run_ranks_some_die(_killed_rank, 2)
    assert codes == [0, -signal.SIGKILL]
    assert out is not None and out["step"] == 1 and out["ranks"] == [1]


def _delayed_rank(rank, world):
    from my_muon_fsdp2_b200.parallel.fault import FaultInjector, RankFailure, guarded_barrier

    import torch.distributed as dist

    inj = FaultInjector(rank, delay_at=(1, 0, 3.0))
    dist.barrier()  # both ranks start the step together, however late either process came up
    try:
        inj.on_step(0)
        guarded_barrier(timeout_s=0.5)
        res = "ok"
    except (RankFailure, RuntimeError):
        res = "timeout"
    # after a detected failure the group is not used again (both ranks simply leave)
    return res


def test_delayed_rank_times_out_monitored_barrier():
    assert run_ranks(_delayed_rank, 2) == "timeout"


def _corrupted(rank, world):
    from my_muon_fsdp2_b200.parallel.fault import FaultInjector, verify_replicas

    torch.manual_seed(0)
    ts = [torch.randn(8, 8), torch.randn(16)]
    if rank == 1:
        FaultInjector.corrupt(ts[1])
    return verify_replicas(ts)


def test_verify_replicas_finds_corruption():
    assert run_ranks(_corrupted, 2) == [1]


def test_step_watchdog_fires():
    from my_muon_fsdp2_b200.parallel.fault import StepWatchdog

    fired = []
    with StepWatchdog(0.1, on_timeout=lambda: fired.append(1)) as w:
        time.sleep(0.3)
    assert w.fired and fired
