"""Shared optimizer plumbing: state allocation, engine access, checkpoint layout helpers."""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch

from ..parallel.dtensor import is_dtensor
from ..parallel.muon_engine import MuonEngine


def zeros_state_like(p: torch.Tensor, fp32_on_cuda: bool = True) -> torch.Tensor:
    """Momentum-style state for ``p``: same layout (a DTensor for DTensor params), fp32 on CUDA.

    CPU parameters keep the parameter dtype, exactly like ``torch.zeros_like(p)`` in the
    reference (optimizer.py:134-136); CUDA parameters get fp32 state because the fused kernels
    accumulate momentum in fp32 (bf16 parameters, fp32 momentum).
    """
    if is_dtensor(p):
        from torch.distributed.tensor import DTensor

        loc = p.to_local()
        dt = torch.float32 if (loc.is_cuda and fp32_on_cuda) else loc.dtype
        z = torch.zeros(loc.shape, dtype=dt, device=loc.device)
        return DTensor.from_local(z, p.device_mesh, p.placements, run_check=False, shape=p.shape,
                                  stride=p.stride())
    dt = torch.float32 if (p.is_cuda and fp32_on_cuda) else p.dtype
    return torch.zeros(p.shape, dtype=dt, device=p.device)


def local_of(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    return t.to_local() if is_dtensor(t) else t


_ENGINES: Dict[Any, MuonEngine] = {}


def default_engine(group=None, comm: str = "auto", split: str = "auto") -> MuonEngine:
    key = (id(group), comm, split)
    eng = _ENGINES.get(key)
    if eng is None:
        eng = MuonEngine(process_group=group, comm=comm, split=split)
        _ENGINES[key] = eng
    return eng


def index_state_dict(opt: torch.optim.Optimizer, extra: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """Standard torch layout {"state": {idx: {...}}, "param_groups": [{..., "params": [idx]}]} + extras.

    The per-parameter entries and group keys are the reference's; parameters are addressed by
    integer index (as torch.optim does) so that the dict can be saved and loaded in a new process.
    """
    index: Dict[int, int] = {}
    groups: List[Dict[str, Any]] = []
    nxt = 0
    for g in opt.param_groups:
        packed = {k: v for k, v in g.items() if k != "params"}
        ids = []
        for p in g["params"]:
            if id(p) not in index:
                index[id(p)] = nxt
                nxt += 1
            ids.append(index[id(p)])
        packed["params"] = ids
        groups.append(packed)
    state = {}
    for g in opt.param_groups:
        for p in g["params"]:
            if p in opt.state and len(opt.state[p]):
                state[index[id(p)]] = dict(opt.state[p])
    out: Dict[str, Any] = {"state": state, "param_groups": groups}
    if extra:
        out.update(extra)
    return out


def load_index_state_dict(opt: torch.optim.Optimizer, sd: Dict[str, Any]) -> None:
    """Inverse of :func:`index_state_dict`; also accepts Parameter-keyed dicts (same process)."""
    params = [p for g in opt.param_groups for p in g["params"]]
    saved_groups = sd["param_groups"]
    if len(saved_groups) != len(opt.param_groups):
        raise ValueError("loaded state dict has a different number of parameter groups")
    flat_saved = [q for g in saved_groups for q in g["params"]]
    if len(flat_saved) != len(params):
        raise ValueError("loaded state dict contains a different number of parameters")
    key_to_param = {}
    for saved, p in zip(flat_saved, params):
        key_to_param[saved if isinstance(saved, int) else id(saved)] = p
    for g, sg in zip(opt.param_groups, saved_groups):
        for k, v in sg.items():
            if k != "params":
                g[k] = v
    opt.state.clear()
    for k, v in sd["state"].items():
        p = key_to_param[k if isinstance(k, int) else id(k)]
        entry = {}
        for name, val in v.items():
            if isinstance(val, torch.Tensor):
                cur = val
                if is_dtensor(p) and not is_dtensor(val):
                    from torch.distributed.tensor import DTensor

                    cur = DTensor.from_local(val.to(p.to_local().device), p.device_mesh, p.placements,
                                             run_check=False, shape=p.shape, stride=p.stride())
                elif not is_dtensor(val):
                    cur = val.to(p.device)
                entry[name] = cur
            else:
                entry[name] = val
        opt.state[p] = entry
