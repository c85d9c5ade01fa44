"""Training-step API (parity with the reference trainers' loop, examples/train_gpt.py:298-402).

``Trainer.train_step(batch)`` is the end-to-end call a user makes: it copies the step's
token batch from (pinned) host memory to the GPU, runs ``grad_accum`` micro-batches of
forward/backward (FSDP2 gradient sync only on the last one), steps every optimizer, clears
gradients and returns the loss as a Python float (one device->host read).
"""
from __future__ import annotations

import os
import time
from typing import Optional, Sequence

import torch
import torch.nn as nn

from ..parallel.fsdp_utils import is_fsdp_module
from ..utils.tracing import nvtx_range


def clip_grad_norm(params, max_norm: float) -> torch.Tensor:
    """``torch.nn.utils.clip_grad_norm_`` for parameter lists that mix sharded DTensor gradients
    (FSDP2 or SymmFSDP shards) with plain replicated ones (the replicated rest of a SymmFSDP
    model): the global 2-norm combines the DTensors' norm (reduced over their mesh) with the
    plain tensors' local norm, and the clip factor scales each gradient in place.  No host
    synchronisation.  Lists of one kind go to PyTorch's function unchanged."""
    grads = [p.grad for p in params if p.grad is not None]
    sharded = [g for g in grads if hasattr(g, "to_local")]
    plain = [g for g in grads if not hasattr(g, "to_local")]
    if not sharded or not plain:
        return torch.nn.utils.clip_grad_norm_(params, max_norm)
    n_sh = torch.nn.utils.get_total_norm(sharded, 2.0)
    if hasattr(n_sh, "full_tensor"):
        n_sh = n_sh.full_tensor()
    n_pl = torch.nn.utils.get_total_norm(plain, 2.0)
    total = torch.sqrt(n_sh.float() ** 2 + n_pl.float().to(n_sh.device) ** 2)
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    torch._foreach_mul_([g.to_local() for g in sharded], coef)
    torch._foreach_mul_(plain, coef.to(plain[0].device))
    return total


class Trainer:
    def __init__(self, model: nn.Module, optimizers: Sequence, grad_accum: int = 1, device=None,
                 step_timer=None, max_grad_norm: Optional[float] = None, time_steps: bool = False,
                 keep_gathered: bool = False, time_phases: bool = False):
        """``max_grad_norm``: clip the global gradient norm before the optimizer steps, as the
        reference trainers do with 1.0 (examples/train_gpt.py:367-371); None disables it.
        ``time_steps``: bracket every step with CUDA events (read by ``last_step_ms`` and
        ``metrics_summary``; no synchronisation inside the step).
        ``keep_gathered``: FSDP2 modules do not reshard after the backward of a non-final
        micro-batch, so the next micro-batch's forward needs no all-gather (FSDP2's
        ``set_reshard_after_backward``; the root module then gathers once per step) at the cost
        of holding the gathered parameters through the accumulation; the last micro-batch
        reshards as usual.
        ``time_phases``: CUDA events between the phases of every step (each micro-batch's
        forward and backward, gradient clipping, the optimizer step); ``phase_ms()`` reads the
        last step's durations.  Events add no work and no synchronisation inside the step."""
        self.model = model
        self.max_grad_norm = max_grad_norm
        self.last_grad_norm: Optional[torch.Tensor] = None
        self.steps = 0
        self.last_metrics: dict = {}
        self.optimizers = list(optimizers)
        self.grad_accum = int(grad_accum)
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.step_timer = step_timer  # optional EventTimer around the optimizer steps
        self.fsdp = is_fsdp_module(model)
        # gradient synchronisation only on the last micro-batch: FSDP2 modules and models whose
        # linears are on the fused collectives (whose rest may be replicated, not FSDP2)
        self.grad_sync = self.fsdp or getattr(model, "_symm_fsdp", None) is not None
        self.keep_gathered = bool(keep_gathered) and self.fsdp and self.grad_accum > 1
        self.time_steps = bool(time_steps) and self.device.type == "cuda"
        self._step_events = None
        self.time_phases = bool(time_phases) and self.device.type == "cuda"
        self._phase_marks: list = []
        self._host_marks: list = []
        self._probes: list = []
        self._clock_probe = self.time_phases and os.environ.get("MMF_CLOCK_PROBE") == "1"
        self._prev_comm: Optional[dict] = None
        ctl = getattr(model, "_symm_fsdp", None)  # fused-collective linears: regather after each step
        if ctl is not None:
            for opt in self.optimizers:
                ctl.attach_optimizer(opt)

    def _micro(self, tokens: torch.Tensor, i: int):
        last = i == self.grad_accum - 1
        if self.grad_sync:
            self.model.set_requires_gradient_sync(last)
        if self.fsdp:
            if self.keep_gathered and i in (0, self.grad_accum - 1):
                # no resharding after the backward of a non-final micro-batch: the next forward
                # finds the parameters still gathered
                self.model.set_reshard_after_backward(last)
        t = tokens[i]
        with nvtx_range(f"trainer/micro_batch_{i}/forward"):
            loss = self.model(t[:, :-1], t[:, 1:]) / self.grad_accum
        self._mark(f"forward_{i}")
        with nvtx_range(f"trainer/micro_batch_{i}/backward"):
            loss.backward()
        self._mark(f"backward_{i}")
        return loss

    def _mark(self, name: str) -> None:
        if self.time_phases:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._phase_marks.append((name, ev))
            # when the host got here: phases whose host time reaches their device time are
            # launch-bound (the GPU waits for the host)
            self._host_marks.append((name, time.perf_counter()))
            if self._clock_probe:
                # diagnostic: the SM clock at this phase boundary (clock_probe kernel, 148 SMs)
                from .._ext import ext

                out = torch.empty(148, 2, dtype=torch.int64, device=self.device)
                ext().clock_probe(out, 200000)
                self._probes.append((name, out))

    def phase_ms(self) -> dict:
        """Device time of each phase of the last step (waits for it); {} unless ``time_phases``.
        The backward phases include the weight-gradient collectives joined at their end."""
        if len(self._phase_marks) < 2:
            return {}
        self._phase_marks[-1][1].synchronize()
        out = {}
        for (_, a), (name, b) in zip(self._phase_marks[:-1], self._phase_marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def step_on_device(self, tokens: torch.Tensor) -> torch.Tensor:
        """One optimizer step on a device batch [grad_accum, micro_bs, seq+1]; returns the loss
        (device tensor, no synchronisation)."""
        if self.time_steps:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record()
        self._phase_marks = []
        self._host_marks = []
        self._probes = []
        self._mark("start")
        total = None
        for i in range(self.grad_accum):
            l = self._micro(tokens, i).detach()
            total = l if total is None else total + l
        if self.max_grad_norm is not None:
            ctl = getattr(self.model, "_symm_fsdp", None)
            if ctl is not None:
                ctl.wait_replicated_grads()  # the norm reads every gradient
            params = [p for p in self.model.parameters() if p.grad is not None]
            self.last_grad_norm = clip_grad_norm(params, self.max_grad_norm)
            self._mark("grad_clip")
        if self.step_timer is not None:
            self.step_timer.start()
        with nvtx_range("trainer/optimizer_step"):
            for opt in self.optimizers:
                opt.step()
        if self.step_timer is not None:
            self.step_timer.stop()
        self._mark("optimizer")
        for opt in self.optimizers:
            opt.zero_grad(set_to_none=True)
        if self.time_steps:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record()
            self._step_events = (t0, t1)
        self.steps += 1
        self.last_metrics = self._metrics(tokens, total)
        return total

    def _metrics(self, tokens: torch.Tensor, loss: torch.Tensor) -> dict:
        """Per-step observability without a device sync: loss / grad norm stay device tensors;
        the Muon engine's exchange statistics and the fused-FSDP state are host values."""
        m = {"step": self.steps, "micro_batches": self.grad_accum,
             "tokens": int(tokens[:, :, 1:].numel()), "loss": loss}
        if self.last_grad_norm is not None:
            m["grad_norm"] = self.last_grad_norm
        if self.step_timer is not None and getattr(self.step_timer, "pairs", None):
            m["optimizer_step_timer"] = self.step_timer
        for k, opt in enumerate(self.optimizers):
            eng = getattr(opt, "_engine", None)
            if eng is not None:
                for key, val in getattr(eng, "last_stats", {}).items():
                    m[f"opt{k}/{key}"] = val
                m[f"opt{k}/cooperative_matrices"] = getattr(eng, "split_count", 0)
        ctl = getattr(self.model, "_symm_fsdp", None)
        if ctl is not None:
            m["symm_fsdp/world"] = ctl.world
            m["symm_fsdp/rs_mode"] = ctl.rs_mode
            m["symm_fsdp/resident_weights"] = sum(1 for f in ctl.full if f is not None)
            m["symm_fsdp/memory_bytes"] = sum(ctl.memory_bytes().values())
            cur = ctl.stats()
            prev = self._prev_comm or {k: 0 for k in cur}
            for k, v in cur.items():  # this step's traffic
                m[f"symm_fsdp/{k}"] = v - prev[k]
            self._prev_comm = cur
        return m

    def last_step_ms(self) -> Optional[float]:
        """Device time of the last step (waits for it); None unless ``time_steps``."""
        if self._step_events is None:
            return None
        t0, t1 = self._step_events
        t1.synchronize()
        return t0.elapsed_time(t1)

    def metrics_summary(self) -> dict:
        """``last_metrics`` with device values read back (synchronises), plus the step time,
        tokens/s and the achieved bandwidth of the step's collectives when they are known."""
        out = {}
        for k, v in self.last_metrics.items():
            if isinstance(v, torch.Tensor):
                out[k] = float(v.detach().float().item())
            elif hasattr(v, "mean_ms"):
                out[k.replace("timer", "ms")] = v.mean_ms()
            else:
                out[k] = v
        if self.device.type == "cuda":  # the monitoring the reference's performance guide suggests
            out["max_memory_allocated_gb"] = torch.cuda.max_memory_allocated(self.device) / 2**30
        ms = self.last_step_ms()
        if ms:
            out["step_ms"] = ms
            out["tokens_per_s"] = out["tokens"] / (ms / 1e3)
            comm = sum(v for k, v in out.items()
                       if isinstance(v, (int, float)) and (k.endswith("exchange_bytes") or k.startswith("symm_fsdp/bytes")))
            out["comm_bytes"] = comm
            out["comm_gbps"] = comm / (ms / 1e3) / 1e9
        return out

    def train_step(self, batch: torch.Tensor) -> float:
        """End-to-end step from a host batch [grad_accum, micro_bs, seq+1] (int64)."""
        tokens = batch.to(self.device, non_blocking=True)
        return float(self.step_on_device(tokens).item())
