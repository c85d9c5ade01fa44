"""Failure detection for multi-rank training (host side) and the device-side error check.

The reference has none (its only robustness code swallows exceptions, hdsp.py:137-139).  Here:

* :class:`Heartbeat` — every rank publishes a timestamp in the rendezvous store from a
  background thread; :meth:`Heartbeat.dead_ranks` / :meth:`Heartbeat.check` find ranks whose
  heartbeat is older than a limit, so the survivors learn of a dead or hung rank *between steps*
  (before their next collective) instead of blocking in it.
* :func:`guarded_barrier` — a barrier with a deadline (gloo ``monitored_barrier`` names the
  missing ranks; when a peer's process died and the barrier fails with a transport error instead,
  the heartbeat names the rank that went quiet; NCCL groups fall back to a heartbeat check +
  barrier).
* :func:`verify_replicas` — detects corrupted/diverged replicated tensors by comparing
  checksums across ranks.
* :class:`StepWatchdog` — fires a callback (default: dump stacks) when a step exceeds a limit.
* :class:`FaultInjector` — host-side injection for tests: raise on a given rank/step, delay a
  rank, stop heart-beating (simulated hang), corrupt a tensor.  Nothing here faults a GPU.
* :func:`check_device` — reads the device error word written by our kernels' bounded waits.
* :func:`init_distributed` — joins a torchrun job with a collective timeout, NCCL async error
  handling and an eagerly created communicator.
"""
from __future__ import annotations

import datetime
import faulthandler
import sys
import threading
import time
from typing import Callable, List, Optional

import torch
import torch.distributed as dist


class RankFailure(RuntimeError):
    """One or more peer ranks stopped making progress."""

    def __init__(self, ranks: List[int], msg: str = ""):
        super().__init__(msg or f"ranks {ranks} stopped responding")
        self.ranks = ranks


class Heartbeat:
    def __init__(self, store: dist.Store, rank: int, world: int, interval_s: float = 0.2, prefix: str = "mmf/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval_s, self.prefix = interval_s, prefix
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def start(self) -> "Heartbeat":
        self.beat()

        def loop():
            while not self._stop.wait(self.interval_s):
                if not self._paused.is_set():
                    try:
                        self.beat()
                    except Exception:
                        return

        self._thread = threading.Thread(target=loop, daemon=True, name="mmf-heartbeat")
        self._thread.start()
        return self

    def pause(self) -> None:  # used by the fault injector to simulate a hung rank
        self._paused.set()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def last_seen(self, r: int) -> Optional[float]:
        try:
            if not self.store.check([self._key(r)]):
                return None
            return float(self.store.get(self._key(r)).decode())
        except Exception:
            return None

    def dead_ranks(self, limit_s: float) -> List[int]:
        now = time.time()
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            t = self.last_seen(r)
            if t is None or now - t > limit_s:
                out.append(r)
        return out

    def check(self, limit_s: float) -> None:
        dead = self.dead_ranks(limit_s)
        if dead:
            raise RankFailure(dead)


def guarded_barrier(timeout_s: float = 30.0, group: Optional[dist.ProcessGroup] = None,
                    heartbeat: Optional[Heartbeat] = None) -> None:
    """Barrier that ends with an error instead of waiting forever."""
    if heartbeat is not None:
        heartbeat.check(timeout_s)
    backend = dist.get_backend(group)
    if backend == "gloo":
        try:
            dist.monitored_barrier(group=group, timeout=datetime.timedelta(seconds=timeout_s), wait_all_ranks=True)
        except RuntimeError as e:
            ranks = _ranks_from_message(str(e))
            if not ranks and heartbeat is not None:
                # a peer whose process died closes its connections: the barrier then fails with a
                # transport error that names no rank, and the heartbeat tells which rank went quiet
                ranks = _quiet_ranks(heartbeat, timeout_s)
            raise RankFailure(ranks, f"barrier failed: {e}") from e
    else:
        dist.barrier(group=group)


def _quiet_ranks(heartbeat: Heartbeat, limit_s: float) -> List[int]:
    """Ranks whose heartbeat is older than ``limit_s``, polled for up to ``2 * limit_s``."""
    end = time.monotonic() + 2.0 * limit_s
    while True:
        dead = heartbeat.dead_ranks(limit_s)
        if dead or time.monotonic() > end:
            return dead
        time.sleep(min(0.05, limit_s / 4))


def _ranks_from_message(msg: str) -> List[int]:
    import re

    m = re.search(r"Ranks? ([0-9][0-9, ]*?) failed", msg)
    if not m:
        return []
    return [int(x) for x in m.group(1).replace(",", " ").split() if x.isdigit()]


@torch.no_grad()
def verify_replicas(tensors, group: Optional[dist.ProcessGroup] = None) -> List[int]:
    """Indices of tensors whose checksum differs across ranks (empty list when consistent)."""
    sums = torch.stack([t.detach().double().sum() + 1e-3 * t.detach().double().abs().sum() for t in tensors])
    sums = sums.to("cuda" if dist.get_backend(group) == "nccl" else "cpu")
    world = dist.get_world_size(group)
    gathered = [torch.empty_like(sums) for _ in range(world)]
    dist.all_gather(gathered, sums, group=group)
    ref = gathered[0]
    bad = set()
    for g in gathered[1:]:
        for i in torch.nonzero(~torch.isclose(g, ref, rtol=1e-9, atol=0.0)).flatten().tolist():
            bad.add(i)
    return sorted(bad)


class StepWatchdog:
    """``with StepWatchdog(60): step()`` — calls ``on_timeout`` if the block runs too long."""

    def __init__(self, limit_s: float, on_timeout: Optional[Callable[[], None]] = None):
        self.limit_s = limit_s
        self.on_timeout = on_timeout or (lambda: faulthandler.dump_traceback(file=sys.stderr, all_threads=True))
        self.fired = False
        self._timer: Optional[threading.Timer] = None

    def _fire(self):
        self.fired = True
        self.on_timeout()

    def __enter__(self):
        self._timer = threading.Timer(self.limit_s, self._fire)
        self._timer.daemon = True
        self._timer.start()
        return self

    def __exit__(self, *exc):
        self._timer.cancel()
        return False


class FaultInjector:
    """Host-side fault injection for tests (never touches a GPU in a harmful way)."""

    def __init__(self, rank: int, raise_at: Optional[tuple] = None, delay_at: Optional[tuple] = None,
                 hang_at: Optional[tuple] = None):
        # each spec is (rank, step) or (rank, step, seconds) for delay
        self.rank, self.raise_at, self.delay_at, self.hang_at = rank, raise_at, delay_at, hang_at

    def on_step(self, step: int, heartbeat: Optional[Heartbeat] = None) -> None:
        if self.raise_at and self.raise_at[0] == self.rank and self.raise_at[1] == step:
            raise RuntimeError(f"injected failure on rank {self.rank} at step {step}")
        if self.delay_at and self.delay_at[0] == self.rank and self.delay_at[1] == step:
            time.sleep(self.delay_at[2])
        if self.hang_at and self.hang_at[0] == self.rank and self.hang_at[1] == step:
            if heartbeat is not None:
                heartbeat.pause()
            time.sleep(self.hang_at[2] if len(self.hang_at) > 2 else 3600)

    @staticmethod
    @torch.no_grad()
    def corrupt(t: torch.Tensor, value: float = 1e3) -> None:
        t.view(-1)[0] += value


def check_device(device: int = 0) -> None:
    """Raise if one of this library's kernels recorded a bounded-wait timeout on ``device``."""
    from .._ext import check_device_error

    check_device_error(device)


def init_distributed(backend: Optional[str] = None, timeout_s: float = 300.0,
                     async_error_handling: bool = True) -> dict:
    """Join the job that ``torchrun`` described in the environment (RANK, WORLD_SIZE, LOCAL_RANK,
    MASTER_ADDR, MASTER_PORT) with failure handling switched on; a plain single process (no RANK)
    joins nothing.  Returns ``{"rank", "world", "local_rank", "device"}``.

    * backend: ``"nccl"`` when CUDA is available, else ``"gloo"``.
    * ``timeout_s`` bounds every collective: a rank that died or hung ends the others' next
      collective with an error instead of a wait forever.
    * ``async_error_handling`` sets ``TORCH_NCCL_ASYNC_ERROR_HANDLING=1`` (unless already set):
      NCCL's watchdog then aborts the communicator and ends the process on a failed or timed-out
      collective, so no GPU stream stays blocked on a dead peer.
    * NCCL groups are bound to this rank's GPU (``device_id``), which creates the communicator
      eagerly: a missing peer fails here, at start-up, not in the first training step.
    """
    import os

    if "RANK" not in os.environ or "WORLD_SIZE" not in os.environ:
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        return {"rank": 0, "world": 1, "local_rank": 0, "device": dev}
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        if async_error_handling:
            os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        kw["device_id"] = dev
    else:
        dev = torch.device("cpu")
    if not dist.is_initialized():
        dist.init_process_group(backend, rank=rank, world_size=world, **kw)
    return {"rank": rank, "world": world, "local_rank": local, "device": dev}
