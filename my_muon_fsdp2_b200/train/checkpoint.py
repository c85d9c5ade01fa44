"""Checkpoint save / resume.

* :func:`save_checkpoint` / :func:`load_checkpoint` write the reference trainer's layout
  ``{"model_state_dict", "optimizer_state_dict", "epoch", "loss"}`` to ``<dir>/muon_<name>.pt``
  (examples/train_gpt.py:569-580) — and, unlike the reference, can load it back (resume).
  FSDP2 models are gathered to full tensors on rank 0 (``full_state_dict``).
* :func:`save_sharded` / :func:`load_sharded` use ``torch.distributed.checkpoint`` (DCP) for
  large FSDP2 models: every rank writes its own shards, and the optimizer state keeps the same
  logical keys (``momentum_buffer``, ``exp_avg``, ...) as the in-memory layout.
"""
from __future__ import annotations

import os
from typing import Any, Dict, List, Optional, Sequence, Union

import torch
import torch.distributed as dist
import torch.nn as nn

Opts = Union[torch.optim.Optimizer, Sequence[torch.optim.Optimizer]]


def _opts(o: Opts) -> List:
    return list(o) if isinstance(o, (list, tuple)) else [o]


def _is_dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def _full_model_sd(model: nn.Module) -> Dict[str, torch.Tensor]:
    from ..parallel.dtensor import is_dtensor

    out = {}
    for k, v in model.state_dict().items():
        out[k] = (v.full_tensor() if is_dtensor(v) else v).detach().cpu()
    return out


def _full_opt_sd(opt) -> Dict[str, Any]:
    from ..parallel.dtensor import is_dtensor

    sd = opt.state_dict()

    def conv(x):
        if isinstance(x, torch.Tensor):
            return (x.full_tensor() if is_dtensor(x) else x).detach().cpu()
        if isinstance(x, dict):
            return {k: conv(v) for k, v in x.items()}
        return x

    return conv(sd)


def checkpoint_path(save_dir: str, name: str) -> str:
    return os.path.join(save_dir, f"muon_{name}.pt")


def save_checkpoint(save_dir: str, name: str, model: nn.Module, optimizer: Opts, epoch: int, loss: float) -> str:
    """Full (gathered) checkpoint in the reference trainer's layout; written by rank 0."""
    opts = _opts(optimizer)
    payload = {
        "model_state_dict": _full_model_sd(model),
        "optimizer_state_dict": _full_opt_sd(opts[0]) if len(opts) == 1 else [_full_opt_sd(o) for o in opts],
        "epoch": epoch,
        "loss": loss,
    }
    path = checkpoint_path(save_dir, name)
    if not _is_dist() or dist.get_rank() == 0:
        os.makedirs(save_dir, exist_ok=True)
        torch.save(payload, path)
    if _is_dist():
        dist.barrier()
    return path


def _shard_like(full: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    from ..parallel.dtensor import is_dtensor

    if is_dtensor(like):
        from torch.distributed.tensor import distribute_tensor

        return distribute_tensor(full.to(like.to_local().device, like.dtype), like.device_mesh, like.placements)
    return full.to(like.device, like.dtype)


def load_checkpoint(path: str, model: nn.Module, optimizer: Optional[Opts] = None) -> Dict[str, Any]:
    """Resume from :func:`save_checkpoint` (works for plain and FSDP2-sharded models)."""
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    cur = model.state_dict()
    new = {k: _shard_like(v, cur[k]) for k, v in ckpt["model_state_dict"].items()}
    model.load_state_dict(new)
    if optimizer is not None:
        opts = _opts(optimizer)
        sds = ckpt["optimizer_state_dict"]
        sds = sds if isinstance(sds, list) else [sds]
        for opt, sd in zip(opts, sds):
            params = [p for g in opt.param_groups for p in g["params"]]
            for idx, entry in sd.get("state", {}).items():
                p = params[idx]
                for k, v in list(entry.items()):
                    if isinstance(v, torch.Tensor) and v.dim() > 0 and v.shape == p.shape:
                        entry[k] = _shard_like(v, p).to(torch.float32 if v.dtype == torch.float32 else v.dtype)
            opt.load_state_dict(sd)
    return {"epoch": ckpt.get("epoch"), "loss": ckpt.get("loss")}


def _encode_extra(extra: Optional[Dict[str, Any]]) -> str:
    # one string leaf: DCP loads only the leaves its template has, and an empty dict has none
    import base64
    import pickle

    return base64.b64encode(pickle.dumps(dict(extra or {}))).decode("ascii")


def _decode_extra(blob: str) -> Dict[str, Any]:
    import base64
    import pickle

    return pickle.loads(base64.b64decode(blob)) if blob else {}


@torch.no_grad()
def _init_optimizer_state(opt: torch.optim.Optimizer) -> None:
    """Create the optimizer's lazily-built state (one step on zero gradients at lr 0), so that
    the load template has every entry the checkpoint holds."""
    if opt.state:
        return
    params = [p for g in opt.param_groups for p in g["params"] if p.requires_grad]
    if any(p.grad is not None for p in params):
        return
    for p in params:
        p.grad = torch.zeros_like(p)
    lrs = [g.get("lr") for g in opt.param_groups]
    for g in opt.param_groups:
        if "lr" in g:
            g["lr"] = 0.0
    opt.step()
    for g, lr in zip(opt.param_groups, lrs):
        if lr is not None:
            g["lr"] = lr
    for p in params:
        p.grad = None


def save_sharded(path: str, model: nn.Module, optimizer: Opts, extra: Optional[Dict[str, Any]] = None) -> None:
    """DCP checkpoint: each rank writes its shards of the model and optimizer state; ``extra``
    (picklable metadata: epoch, step, ...) is stored alongside."""
    import torch.distributed.checkpoint as dcp

    state = {"model": model.state_dict(), "optim": [o.state_dict() for o in _opts(optimizer)],
             "extra": _encode_extra(extra)}
    dcp.save(state, checkpoint_id=path)


def load_sharded(path: str, model: nn.Module, optimizer: Opts) -> Dict[str, Any]:
    """Load a :func:`save_sharded` checkpoint into ``model`` / ``optimizer`` (re-sharded to the
    current layout by DCP) and return its ``extra`` metadata."""
    import torch.distributed.checkpoint as dcp

    opts = _opts(optimizer)
    for o in opts:
        _init_optimizer_state(o)
    state = {"model": model.state_dict(), "optim": [o.state_dict() for o in opts], "extra": ""}
    dcp.load(state, checkpoint_id=path)
    model.load_state_dict(state["model"])
    for o, sd in zip(opts, state["optim"]):
        o.load_state_dict(sd)
    return _decode_extra(state["extra"])
