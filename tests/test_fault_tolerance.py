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


def _init_entry(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from my_muon_fsdp2_b200.parallel.fault import init_distributed

    info = init_distributed(backend="gloo", timeout_s=2.0)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t)
    res = {"info": info, "sum": float(t), "backend": dist.get_backend()}
    # rank 1 leaves without taking the next collective: rank 0's all_reduce must end with an
    # error once the group's timeout has passed, not wait forever
    if rank == 0:
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(1))
            res["late"] = "completed"
        except RuntimeError:
            res["late"] = round(time.time() - t0, 1)
        torch.save(res, path)
    else:
        time.sleep(5.0)
    dist.destroy_process_group()


def test_init_distributed_joins_with_a_collective_timeout(tmp_path):
    import torch.multiprocessing as mp

    from tests.conftest import free_port

    for attempt in range(3):
        path = str(tmp_path / f"r{attempt}.pt")
        try:
            mp.spawn(_init_entry, args=(2, free_port(), path), nprocs=2, join=True)
        except mp.ProcessRaisedException as e:
            if attempt < 2 and "address already in use" in str(e).lower():
                continue
            raise
        break
    res = torch.load(path, weights_only=False)
    assert res["backend"] == "gloo" and res["sum"] == 3.0
    assert res["info"]["rank"] == 0 and res["info"]["world"] == 2 and str(res["info"]["device"]) == "cpu"
    assert res["late"] != "completed" and res["late"] < 4.5


def test_init_distributed_single_process(monkeypatch):
    from my_muon_fsdp2_b200.parallel.fault import init_distributed

    monkeypatch.delenv("RANK", raising=False)
    info = init_distributed()
    assert info["rank"] == 0 and info["world"] == 1 and not dist.is_initialized()
