"""Muon step engine: momentum + Newton–Schulz + parameter update for plain or FSDP2-sharded params.

This is the B200 replacement of the reference's "NS replication" step
(``src/muon_fsdp/fsdp.py:253-450``: per-parameter all-gather of the raw gradient, identical NS on
every rank, row slice).  Instead of replicating the NS work ``world_size`` times, each matrix is
given one *owner* rank (longest-processing-time-first assignment on its NS FLOP count), so the
chain runs once per matrix and the ranks split the FLOPs:

1. every rank updates the momentum of its local row shards (``muon_prep`` kernel: momentum,
   Nesterov, coupled weight decay, bf16 cast, per-matrix sum of squares) and writes the bf16
   NS input for matrix *j* into the staging segment of ``owner(j)``;
2. the per-matrix partial sums of squares are all-reduced (a few hundred floats);
3. the staged shards reach their owners (``comm="nccl"``: one ``all_to_all_single`` for all
   matrices; ``comm="p2p"``: the owner's assembly kernel reads the shards straight out of the
   peers' symmetric-memory buffers over NVLink);
4. each owner stacks its matrices by shape and runs the batched tcgen05 chain; the last GEMM's
   epilogue scatters every rank's row shard of the orthogonalised update into that rank's
   return segment (local buffer for NCCL, the peer's symmetric buffer for P2P);
5. after the return exchange each rank applies ``p = (1 - lr*wd) * p - lr_eff * O`` to its shard
   (``muon_prep`` in direct-apply mode).  With ``comm="p2p"`` and parameters that live in
   peer-mapped storage (the shards of the fused FSDP linears), the owner's final epilogue
   applies this update straight into every rank's parameter shard instead, and there is no
   return buffer or local apply for them.

Unsharded (plain) parameters, or a world of one, take the local path: the momentum kernel
writes directly into the NS workspace and the last GEMM epilogue updates the parameters.

CPU tensors (gloo process groups, tests) run the same schedule with PyTorch math in fp32.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops.newton_schulz import NS_COEFFICIENTS, NS_EPS, _ns_torch
from .comm import chunk_offset, chunk_rows
from .dtensor import is_dtensor
from ..utils.tracing import nvtx_range
from ..optim.errors import SparseGradientError

MODE_COPY, MODE_EMA, MODE_HEAVYBALL = 0, 1, 2


@dataclass
class MuonHyper:
    """Momentum form shared by one engine call (one parameter group)."""

    mode: int = MODE_EMA  # EMA (lerp) or heavy-ball (buf = mu*buf + g)
    momentum: float = 0.95
    nesterov: bool = False
    wd_coupled: float = 0.0  # g <- g + wd * p before the momentum update
    ns_steps: int = 5


@dataclass
class MuonTask:
    """One parameter: its update is p <- decay * p - lr_eff * U."""

    param: torch.Tensor
    grad: torch.Tensor
    buf: Optional[torch.Tensor]  # fp32 momentum (local shard) or None in copy mode
    lr_eff: float
    decay: float = 1.0
    orthogonalize: bool = True
    # filled by the engine
    local_param: Optional[torch.Tensor] = field(default=None, repr=False)
    local_grad: Optional[torch.Tensor] = field(default=None, repr=False)


def ns_flops(rows: int, cols: int, steps: int) -> float:
    m, n = min(rows, cols), max(rows, cols)
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)


def assign_owners(costs: Sequence[float], world: int) -> List[int]:
    """Longest-processing-time-first: biggest matrix to the least-loaded rank (ties -> lowest rank)."""
    load = [0.0] * world
    owners = [0] * len(costs)
    for j in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda k: (load[k], k))
        owners[j] = r
        load[r] += costs[j]
    return owners


# Relative throughputs of the schedule cost model (only their ratio matters).
_GEMM_FLOPS = 1.4e15   # sustained bf16 tensor-core rate
_LINK_BPS = 7.0e11     # NVLink bytes/s per direction per GPU


def split_eligible(rows: int, cols: int, world: int) -> bool:
    """The cooperative schedule takes wide matrices whose row shards are whole GEMM tiles."""
    return world > 1 and rows <= cols and rows % (128 * world) == 0 and rows % 256 == 0 and cols % 256 == 0


def select_split(shapes: Sequence[Tuple[int, int]], world: int, steps: int) -> List[int]:
    """Per-shape schedule choice.  Owner-computes runs each matrix's whole chain on one rank
    (makespan = LPT load of the busiest rank); the cooperative schedule splits one matrix's
    chain over all ranks (FLOPs / world, plus two all-gathers per iteration).  Matrices move to
    the cooperative schedule, largest first, while that lowers the predicted step time — in
    practice the ones bigger than the average per-rank load, e.g. 8192 x 28672 among
    4096-wide layers."""
    costs = [ns_flops(r, c, steps) / _GEMM_FLOPS for r, c in shapes]

    def makespan(idx):
        if not idx:
            return 0.0
        owners = assign_owners([costs[i] for i in idx], world)
        load = [0.0] * world
        for i, o in zip(idx, owners):
            load[o] += costs[i]
        return max(load)

    def split_time(i):
        r, c = shapes[i]
        comm = steps * 2.0 * (r * c + r * r) * (world - 1) / world / _LINK_BPS
        return costs[i] / world + comm

    rest = list(range(len(shapes)))
    chosen: List[int] = []
    best = makespan(rest)
    for i in sorted(rest, key=lambda k: -costs[k]):
        if not split_eligible(shapes[i][0], shapes[i][1], world):
            continue
        cand = [k for k in rest if k != i]
        t = makespan(cand) + sum(split_time(k) for k in chosen + [i])
        if t < best:
            best, rest = t, cand
            chosen.append(i)
        else:
            break
    return sorted(chosen)


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if is_dtensor(t) else t


def _as2d(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 2:
        return t
    if t.dim() <= 1:
        return t.reshape(1, -1)
    return t.reshape(t.shape[0], -1)


class MuonEngine:
    """Executes Muon steps for lists of :class:`MuonTask` (see module docstring)."""

    def __init__(self, process_group: Optional[dist.ProcessGroup] = None, comm: str = "auto",
                 max_workspace_bytes: int = 8 << 30, split: str = "auto", direct_update: bool = True):
        if comm not in ("auto", "nccl", "p2p"):
            raise ValueError(f"comm must be 'auto', 'nccl' or 'p2p', got {comm!r}")
        if split not in ("auto", "never", "always"):
            raise ValueError(f"split must be 'auto', 'never' or 'always', got {split!r}")
        self.group = process_group
        self.comm = comm
        self.split = split
        self.split_count = 0  # matrices of the last step that took the cooperative schedule
        self.max_workspace_bytes = int(max_workspace_bytes)
        # comm="p2p": write updates straight into parameters that live in peer-mapped storage
        self.direct_update = bool(direct_update)
        self._direct_agreed: Dict[tuple, List[bool]] = {}
        self._p2p = None
        self.last_stats: Dict[str, float] = {}

    # ------------------------------------------------------------------ helpers
    def _world(self, tasks: Sequence[MuonTask]) -> Tuple[int, int, Optional[dist.ProcessGroup]]:
        sharded = [t for t in tasks if is_dtensor(t.param)]
        if not sharded:
            return 1, 0, None
        group = self.group
        if group is None:
            mesh = sharded[0].param.device_mesh
            group = mesh.get_group(mesh.ndim - 1) if mesh.ndim > 1 else mesh.get_group()
        return dist.get_world_size(group), dist.get_rank(group), group

    # ------------------------------------------------------------------ public
    @torch.no_grad()
    def step(self, tasks: Sequence[MuonTask], hp: MuonHyper) -> None:
        tasks = [t for t in tasks if t.grad is not None]
        if not tasks:
            return
        for t in tasks:
            if t.grad.is_sparse:
                raise SparseGradientError("Muon does not support sparse gradients")
            t.local_param = _local(t.param)
            t.local_grad = _local(t.grad)
        world, rank, group = self._world(tasks)
        is_cuda = tasks[0].local_param.is_cuda
        elementwise = [t for t in tasks if not (t.orthogonalize and t.param.dim() == 2)]
        matrices = [t for t in tasks if t.orthogonalize and t.param.dim() == 2]
        if elementwise:
            with nvtx_range("muon/elementwise"):
                self._elementwise(elementwise, hp, is_cuda)
        if not matrices:
            return
        sharded = [t for t in matrices if is_dtensor(t.param)]
        local = [t for t in matrices if not is_dtensor(t.param)]
        if world == 1:
            local = local + sharded
            sharded = []
        if local:
            with nvtx_range("muon/local"):
                if is_cuda:
                    self._local_cuda(local, hp)
                else:
                    self._local_cpu(local, hp)
        if sharded and world > 1 and self.split != "never":
            shp = [tuple(t.param.shape) for t in sharded]
            if self.split == "always":
                pick = [i for i, (r, c) in enumerate(shp) if split_eligible(r, c, world)]
            else:
                pick = select_split(shp, world, hp.ns_steps)
            for i in pick:
                with nvtx_range("muon/cooperative_chain"):
                    self._split_chain(sharded[i], hp, world, rank, group, is_cuda)
            self.split_count = len(pick)
            sharded = [t for i, t in enumerate(sharded) if i not in set(pick)]
        if sharded:
            if is_cuda and self._use_p2p(group):
                with nvtx_range("muon/owner_computes_p2p"):
                    self._sharded_p2p(sharded, hp, world, rank, group)
            else:
                with nvtx_range("muon/owner_computes_nccl"):
                    self._sharded(sharded, hp, world, rank, group, is_cuda)

    def _use_p2p(self, group) -> bool:
        if self.comm == "nccl":
            return False
        from .symm import p2p_supported

        ok = p2p_supported(group)
        if self.comm == "p2p" and not ok:
            raise RuntimeError("comm='p2p' needs an NCCL process group on CUDA devices")
        return ok

    # ------------------------------------------------------------------ elementwise (no NS)
    def _elementwise(self, tasks: List[MuonTask], hp: MuonHyper, is_cuda: bool) -> None:
        if is_cuda:
            from .._ext import ext

            E = ext()
            for key, ts in _group_by(tasks, lambda t: (t.local_grad.dtype, t.local_param.dtype)).items():
                grads = [_as2d(t.local_grad.contiguous()) for t in ts]
                params = [_as2d(t.local_param) for t in ts]
                bufs = [_as2d(t.buf) for t in ts] if hp.mode != MODE_COPY else []
                E.muon_prep(grads, bufs, params, None, [], [], [], [0], [_decay_float(t.decay) for t in ts],
                            [-t.lr_eff for t in ts], hp.mode, hp.nesterov, hp.momentum, hp.wd_coupled, None)
            return
        for t in tasks:
            u = _momentum_torch(t, hp)
            p = t.local_param
            _decay_(p, t.decay)
            p.add_(u.to(p.dtype).reshape(p.shape), alpha=-t.lr_eff)

    # ------------------------------------------------------------------ local paths
    def _local_cpu(self, tasks: List[MuonTask], hp: MuonHyper) -> None:
        for t in tasks:
            u = _momentum_torch(t, hp)
            o = _ns_torch(u, hp.ns_steps)
            p = t.local_param
            _decay_(p, t.decay)
            p.add_(o.to(p.dtype), alpha=-t.lr_eff)

    def _local_cuda(self, tasks: List[MuonTask], hp: MuonHyper) -> None:
        from .._ext import ext
        from ..ops.ns_cuda import round_up, run_ns_group, wide_shape

        E = ext()
        dev = tasks[0].local_param.device
        groups = _group_by(tasks, lambda t: (tuple(t.local_param.shape), t.local_grad.dtype, t.local_param.dtype))
        for (shape, gdt, pdt), ts in groups.items():
            rows, cols = shape
            mw, nw, tall = wide_shape(rows, cols)
            Mp, Np = round_up(mw), round_up(nw)
            per = 2 * Mp * Np * 2 + 2 * Mp * Mp * 2
            chunk = max(1, min(len(ts), self.max_workspace_bytes // max(per, 1)))
            for c0 in range(0, len(ts), chunk):
                sub = ts[c0:c0 + chunk]
                B = len(sub)
                padded = (Mp != mw) or (Np != nw)
                X0 = (torch.zeros if padded else torch.empty)(B, Mp, Np, dtype=torch.bfloat16, device=dev)
                sumsq = torch.zeros(B, dtype=torch.float32, device=dev)
                grads = [t.local_grad.contiguous() for t in sub]
                params = [t.local_param for t in sub]
                bufs = [t.buf for t in sub] if hp.mode != MODE_COPY else []
                E.muon_prep(grads, bufs, params if hp.wd_coupled != 0 else [], X0,
                            [b * Mp * Np for b in range(B)], [0] * B, [int(tall)] * B, [Np], [], [], hp.mode,
                            hp.nesterov, hp.momentum, hp.wd_coupled, sumsq)
                s = torch.empty(B, dtype=torch.float32, device=dev)
                s2 = torch.empty_like(s)
                E.ns_scale(sumsq, B, 1, NS_EPS, s, s2)
                ptrs = E.ptr_table(params)
                pvec = _decay_vec([t.decay for t in sub], dev)
                vvec = _h2d([-t.lr_eff for t in sub], torch.float32, dev)
                run_ns_group(X0, s, s2, hp.ns_steps, ptrs, cols, pdt == torch.float32, tall, mw, nw,
                             p_scale=1.0, v_scale=1.0, p_scale_vec=pvec, v_scale_vec=vvec)

    # ------------------------------------------------------------------ cooperative schedule
    def _split_chain(self, t: MuonTask, hp: MuonHyper, world: int, rank: int, group: dist.ProcessGroup,
                     is_cuda: bool) -> None:
        """One wide matrix X (m x n, m <= n, row-sharded) orthogonalised by all ranks together.
        Rank r owns rows R_r of every iterate; per quintic iteration:

            all-gather X               (every rank needs all of X for its Gram rows)
            A_r = X_r X^T              rows R_r of the Gram matrix (x s^2 on iteration 0)
            all-gather A
            B_r = c A_r A + b A_r      rows R_r of b A + c A^2
            X'_r = B_r X + a X_r       (x s on iteration 0); the last one is written straight
                                       into the parameter shard as p = decay p - lr X'_r

        Each rank does 1/world of the chain's FLOPs; the all-gathers move m n + m^2 elements
        per iteration.  Same algebra as ``newton_schulz_reference`` (fp64 oracle)."""
        a, b, c = NS_COEFFICIENTS
        m, n = t.param.shape
        mr = m // world
        p = t.local_param
        dev = p.device
        if not is_cuda:
            u = _momentum_torch(t, hp).float()
            ss = (u * u).sum().reshape(1)
            dist.all_reduce(ss, group=group)
            X = torch.cat(_gather_list(u.contiguous(), world, group)) / (ss.sqrt() + NS_EPS)
            for it in range(hp.ns_steps):
                if it:
                    X = torch.cat(_gather_list(Xr.contiguous(), world, group))
                Xr = X[rank * mr:(rank + 1) * mr]
                Ar = Xr @ X.t()
                A = torch.cat(_gather_list(Ar.contiguous(), world, group))
                Br = b * Ar + c * (Ar @ A)
                Xr = a * Xr + Br @ X
            _decay_(p, t.decay)
            p.add_(Xr.to(p.dtype), alpha=-t.lr_eff)
            return
        from .._ext import ext

        E = ext()
        Xa = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        Xb = torch.empty_like(Xa)
        Ar = torch.empty(mr, m, dtype=torch.bfloat16, device=dev)
        Af = torch.empty(m, m, dtype=torch.bfloat16, device=dev)
        Br = torch.empty_like(Ar)
        sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        E.muon_prep([t.local_grad.contiguous()], [t.buf] if hp.mode != MODE_COPY else [],
                    [p] if hp.wd_coupled != 0 else [], Xa, [rank * mr * n], [0], [0], [n], [], [], hp.mode,
                    hp.nesterov, hp.momentum, hp.wd_coupled, sumsq)
        parts = torch.empty(world, 1, dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(parts, sumsq, group=group)
        sc = torch.empty(1, dtype=torch.float32, device=dev)
        sc2 = torch.empty_like(sc)
        E.ns_scale(parts, 1, world, NS_EPS, sc, sc2)
        X, Xn = Xa, Xb
        for it in range(hp.ns_steps):
            first = it == 0
            Xr = X[rank * mr:(rank + 1) * mr]
            dist.all_gather_into_tensor(X, Xr, group=group)
            E.tc_gemm_ws(Xr.view(1, mr, n), X.view(1, m, n), False, Ar.view(1, mr, m), None, sc2 if first else None,
                         1.0, None, 0.0, False)
            dist.all_gather_into_tensor(Af, Ar, group=group)
            E.tc_gemm_ws(Ar.view(1, mr, m), Af.view(1, m, m), False, Br.view(1, mr, m), Ar.view(1, mr, m), None, c,
                         None, b, False)
            if it == hp.ns_steps - 1:
                if not p.is_contiguous():
                    raise RuntimeError("MuonEngine: the cooperative schedule needs contiguous parameter shards")
                E.tc_gemm_out(Br.view(1, mr, m), X.view(1, m, n), True, Xr.view(1, mr, n), sc if first else None, 1.0,
                              sc if first else None, a, E.ptr_table([p]), 1, None, n, p.dtype == torch.float32,
                              False, mr, n, _decay_vec([t.decay], dev), 1.0,
                              torch.full((1,), -t.lr_eff, dtype=torch.float32, device=dev), 1.0)
            else:
                Xnr = Xn[rank * mr:(rank + 1) * mr]
                E.tc_gemm_ws(Br.view(1, mr, m), X.view(1, m, n), True, Xnr.view(1, mr, n), Xr.view(1, mr, n),
                             sc if first else None, 1.0, sc if first else None, a, False)
                X, Xn = Xn, X

    # ------------------------------------------------------------------ sharded path
    def _sharded(self, tasks: List[MuonTask], hp: MuonHyper, world: int, rank: int,
                 group: dist.ProcessGroup, is_cuda: bool) -> None:
        n = len(tasks)
        shapes = [tuple(t.param.shape) for t in tasks]
        owners = assign_owners([ns_flops(r, c, hp.ns_steps) for r, c in shapes], world)
        rows_of = [chunk_rows(r, world) for r, _ in shapes]
        for j, t in enumerate(tasks):
            if t.local_param.shape[0] != rows_of[j][rank]:
                raise RuntimeError(
                    "MuonEngine expects FSDP2 Shard(0) parameters laid out like torch.chunk "
                    f"(param {j}: local rows {t.local_param.shape[0]} != {rows_of[j][rank]})")
        owned = [[j for j in range(n) if owners[j] == o] for o in range(world)]
        # element counts of shard (j, r)
        cnt = [[rows_of[j][r] * shapes[j][1] for r in range(world)] for j in range(n)]
        dev = tasks[0].local_param.device
        xdtype = torch.bfloat16 if is_cuda else torch.float32
        # ---- 1. local momentum into the send layout [dest][j in owned(dest)][my rows x cols]
        send_split = [sum(cnt[j][rank] for j in owned[d]) for d in range(world)]
        send = torch.empty(sum(send_split), dtype=xdtype, device=dev)
        send_off: Dict[int, int] = {}
        off = 0
        for d in range(world):
            for j in owned[d]:
                send_off[j] = off
                off += cnt[j][rank]
        sumsq = torch.zeros(n, dtype=torch.float32, device=dev)
        if is_cuda:
            self._cuda_local_momentum(tasks, hp, send, send_off, sumsq)
        else:
            for j, t in enumerate(tasks):
                u = _momentum_torch(t, hp).float()
                sumsq[j] = (u * u).sum()
                send[send_off[j]:send_off[j] + cnt[j][rank]].copy_(u.reshape(-1))
        # ---- 2. global Frobenius norms (CUDA: gather the per-rank partials and sum them in rank
        #      order on the owner, exactly like the P2P path, so both exchanges agree bit for bit)
        parts = None
        if is_cuda:
            parts = torch.empty(world, n, dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(parts, sumsq, group=group)
        else:
            dist.all_reduce(sumsq, group=group)
        # ---- 3. shards -> owners
        recv_split = [sum(cnt[j][r] for j in owned[rank]) for r in range(world)]
        recv = torch.empty(sum(recv_split), dtype=xdtype, device=dev)
        dist.all_to_all_single(recv, send, recv_split, send_split, group=group)
        recv_base = [sum(recv_split[:r]) for r in range(world)]
        # position of shard (j, r) inside recv
        shard_at: Dict[Tuple[int, int], int] = {}
        for r in range(world):
            o = recv_base[r]
            for j in owned[rank]:
                shard_at[(j, r)] = o
                o += cnt[j][r]
        # ---- 4. NS on owned matrices; results scattered into the return layout
        #      back layout: [dest d][j in owned(me)][rows_d(j) x cols]
        back_split = [sum(cnt[j][d] for j in owned[rank]) for d in range(world)]
        back = torch.empty(sum(back_split), dtype=xdtype, device=dev)
        back_base = [sum(back_split[:d]) for d in range(world)]
        back_at: Dict[Tuple[int, int], int] = {}
        for d in range(world):
            o = back_base[d]
            for j in owned[rank]:
                back_at[(j, d)] = o
                o += cnt[j][d]
        if owned[rank]:
            if is_cuda:
                self._cuda_owner_ns(tasks, hp, owned[rank], shapes, rows_of, cnt, world, recv, shard_at, back,
                                    back_at, parts)
            else:
                for j in owned[rank]:
                    rws, cls = shapes[j]
                    full = torch.cat([recv[shard_at[(j, r)]:shard_at[(j, r)] + cnt[j][r]].view(rows_of[j][r], cls)
                                      for r in range(world)])
                    o = _ns_torch(full, hp.ns_steps)
                    for d in range(world):
                        r0 = chunk_offset(rws, world, d)
                        back[back_at[(j, d)]:back_at[(j, d)] + cnt[j][d]].copy_(
                            o[r0:r0 + rows_of[j][d]].reshape(-1))
        # ---- 5. updates back to the shard holders and apply
        ret_split = [sum(cnt[j][rank] for j in owned[o]) for o in range(world)]
        ret = torch.empty(sum(ret_split), dtype=xdtype, device=dev)
        dist.all_to_all_single(ret, back, ret_split, back_split, group=group)
        ret_at: Dict[int, int] = {}
        o_ = 0
        for o in range(world):
            for j in owned[o]:
                ret_at[j] = o_
                o_ += cnt[j][rank]
        if is_cuda:
            self._cuda_apply(tasks, ret, ret_at, cnt, rank)
        else:
            for j, t in enumerate(tasks):
                p = t.local_param
                u = ret[ret_at[j]:ret_at[j] + cnt[j][rank]].view(p.shape)
                _decay_(p, t.decay)
                p.add_(u.to(p.dtype), alpha=-t.lr_eff)
        self.last_stats = {"matrices": float(n), "owned": float(len(owned[rank])),
                           "exchange_bytes": float((send.numel() + ret.numel()) * send.element_size())}

    # ------------------------------------------------------------------ sharded, P2P
    def _sharded_p2p(self, tasks: List[MuonTask], hp: MuonHyper, world: int, rank: int,
                     group: dist.ProcessGroup) -> None:
        """Same schedule as :meth:`_sharded`, with the exchange done by our kernels over NVLink:
        momentum -> own symmetric buffer; barrier (+ partial norms to every peer); owner assembly
        reads peer shards (P2P loads); final NS epilogue stores each rank's rows into that rank's
        buffer, or for parameters in peer-mapped storage applies the update straight into that
        rank's parameter shard (P2P loads and stores); barrier; local apply of the rest."""
        from .._ext import ext
        from ..ops.ns_cuda import round_up, run_ns_group, wide_shape
        from .symm import workspace_for

        E = ext()
        n = len(tasks)
        dev = tasks[0].local_param.device
        shapes = [tuple(t.param.shape) for t in tasks]
        owners = assign_owners([ns_flops(r, c, hp.ns_steps) for r, c in shapes], world)
        rows_of = [chunk_rows(r, world) for r, _ in shapes]
        for j, t in enumerate(tasks):
            if t.local_param.shape[0] != rows_of[j][rank]:
                raise RuntimeError("MuonEngine expects FSDP2 Shard(0) parameters laid out like torch.chunk")
        cnt = [[rows_of[j][r] * shapes[j][1] for r in range(world)] for j in range(n)]
        off = [[0] * n for _ in range(world)]
        for r in range(world):
            o = 0
            for j in range(n):
                off[r][j] = o
                o += cnt[j][r]
        total = max(sum(cnt[j][r] for j in range(n)) for r in range(world))
        sw = workspace_for(group, dev)
        sw.ensure(total, n)
        # 1. momentum of local shards -> own symmetric buffer; partial sums of squares
        part = torch.zeros(n, dtype=torch.float32, device=dev)
        idx = [j for j in range(n) if cnt[j][rank] > 0]
        for key, js in _group_by(idx, lambda j: (tasks[j].local_grad.dtype, tasks[j].local_param.dtype)).items():
            grads = [tasks[j].local_grad.contiguous() for j in js]
            params = [tasks[j].local_param for j in js]
            bufs = [tasks[j].buf for j in js] if hp.mode != MODE_COPY else []
            sub = torch.zeros(len(js), dtype=torch.float32, device=dev)
            E.muon_prep(grads, bufs, params if hp.wd_coupled != 0 else [], sw.buf, [off[rank][j] for j in js],
                        [0] * len(js), [0] * len(js), [shapes[j][1] for j in js], [], [], hp.mode, hp.nesterov,
                        hp.momentum, hp.wd_coupled, sub)
            part.index_copy_(0, _h2d(js, torch.int64, dev), sub)
        # parameters in peer-mapped storage (the fused FSDP shards): the owner's final epilogue
        # applies p <- decay p - lr_eff O straight into every rank's shard of them
        direct = self._direct_targets(tasks, rows_of, group, dev)
        # 2. barrier: every rank's shards are in place; all partial norms delivered to all ranks
        sw.barrier(payload=part)
        rows_ssq = sw.payload_rows()  # [world, n]
        mine = [j for j in range(n) if owners[j] == rank]
        groups = _group_by(mine, lambda j: (wide_shape(*shapes[j])[:2],
                                            tasks[j].local_param.dtype if direct[j] is not None else None))
        for ((mw, nw), direct_dtype), js in groups.items():
            Mp, Np = round_up(mw), round_up(nw)
            per = 2 * Mp * Np * 2 + 2 * Mp * Mp * 2
            chunk = max(1, min(len(js), self.max_workspace_bytes // max(per, 1)))
            for c0 in range(0, len(js), chunk):
                sub_js = js[c0:c0 + chunk]
                tall_group = any(shapes[j][0] > shapes[j][1] for j in sub_js)
                B = len(sub_js)
                padded = (Mp != mw) or (Np != nw)
                X0 = (torch.zeros if padded else torch.empty)(B, Mp, Np, dtype=torch.bfloat16, device=dev)
                srcs, offs, row0, trs = [], [], [], []
                for b, j in enumerate(sub_js):
                    rws, cls = shapes[j]
                    for r in range(world):
                        if rows_of[j][r] == 0:
                            continue
                        # 3. P2P loads: the assembly kernel reads rank r's shard in place
                        srcs.append(sw.peer_view(r, off[r][j], (rows_of[j][r], cls)))
                        offs.append(b * Mp * Np)
                        row0.append(chunk_offset(rws, world, r))
                        trs.append(int(rws > cls))
                E.muon_prep(srcs, [], [], X0, offs, row0, trs, [Np], [], [], MODE_COPY, False, 0.0, 0.0, None)
                jt = _h2d(sub_js, torch.int64, dev)
                ssq = rows_ssq.index_select(1, jt).contiguous()  # [world, B]
                s = torch.empty(B, dtype=torch.float32, device=dev)
                s2 = torch.empty_like(s)
                E.ns_scale(ssq, B, world, NS_EPS, s, s2)
                addrs, meta = [], []
                for j in sub_js:
                    rws, cls = shapes[j]
                    for d in range(world):
                        # 4. P2P stores: rows of rank d go straight into rank d's parameter shard
                        #    (direct) or into rank d's buffer
                        addrs.append(direct[j][d] if direct_dtype is not None else sw.peer_addr(d, off[d][j]))
                    meta += [cls, int(rws > cls), (rws + world - 1) // world]
                ptrs = _h2d(addrs, torch.int64, dev)
                meta_t = _h2d(meta, torch.int64, dev)
                if direct_dtype is not None:
                    pvec = _decay_vec([tasks[j].decay for j in sub_js], dev)
                    vvec = _h2d([-tasks[j].lr_eff for j in sub_js], torch.float32, dev)
                    run_ns_group(X0, s, s2, hp.ns_steps, ptrs, 0, direct_dtype == torch.float32, False, mw, nw,
                                 p_scale=1.0, v_scale=1.0, p_scale_vec=pvec, v_scale_vec=vvec, nseg=world,
                                 out_meta=meta_t, transposed_dest=tall_group)
                else:
                    run_ns_group(X0, s, s2, hp.ns_steps, ptrs, 0, False, False, mw, nw, p_scale=0.0, v_scale=1.0,
                                 nseg=world, out_meta=meta_t, transposed_dest=tall_group)
        # 5. barrier: all owners' results have landed (parameters and buffers)
        sw.barrier()
        # 6. local apply from the own buffer (matrices not updated in place by their owner)
        idx = [j for j in idx if direct[j] is None]
        for key, js in _group_by(idx, lambda j: tasks[j].local_param.dtype).items():
            srcs = [sw.peer_view(rank, off[rank][j], tuple(tasks[j].local_param.shape)) for j in js]
            params = [tasks[j].local_param for j in js]
            E.muon_prep(srcs, [], params, None, [], [], [], [0], [_decay_float(tasks[j].decay) for j in js],
                        [-tasks[j].lr_eff for j in js], MODE_COPY, False, 0.0, 0.0, None)
        self.last_stats = {"matrices": float(n), "owned": float(len(mine)), "exchange_bytes": float(2 * 2 * total),
                           "comm": "p2p", "direct_updates": float(sum(d is not None for d in direct))}

    def _direct_targets(self, tasks: List[MuonTask], rows_of, group: dist.ProcessGroup,
                        dev: torch.device) -> List[Optional[List[int]]]:
        """Per matrix, the address of every rank's parameter shard when the parameters live in
        peer-mapped storage of ``group`` with equal shards (else None).  All ranks must agree:
        the decision is checked with one collective the first time a parameter layout is seen."""
        from .symm import peer_param_addrs

        out: List[Optional[List[int]]] = []
        for j, t in enumerate(tasks):
            lp = t.local_param
            addrs = None
            if self.direct_update and lp.dtype in (torch.bfloat16, torch.float32) and len(set(rows_of[j])) == 1:
                addrs = peer_param_addrs(lp, group)
            out.append(addrs)
        key = tuple((t.local_param.data_ptr(), a is not None) for t, a in zip(tasks, out))
        agreed = self._direct_agreed.get(key)
        if agreed is None:
            flags = torch.tensor([int(a is not None) for a in out], dtype=torch.int32, device=dev)
            dist.all_reduce(flags, op=dist.ReduceOp.MIN, group=group)
            agreed = [bool(f) for f in flags.tolist()]
            self._direct_agreed[key] = agreed
        return [a if ok else None for a, ok in zip(out, agreed)]

    # ---- CUDA pieces of the sharded path
    def _cuda_local_momentum(self, tasks, hp, send, send_off, sumsq) -> None:
        from .._ext import ext

        E = ext()
        idx = list(range(len(tasks)))
        for key, js in _group_by(idx, lambda j: (tasks[j].local_grad.dtype, tasks[j].local_param.dtype)).items():
            live = [j for j in js if tasks[j].local_param.numel() > 0]
            if not live:
                continue
            grads = [tasks[j].local_grad.contiguous() for j in live]
            params = [tasks[j].local_param for j in live]
            bufs = [tasks[j].buf for j in live] if hp.mode != MODE_COPY else []
            part = torch.zeros(len(live), dtype=torch.float32, device=send.device)
            E.muon_prep(grads, bufs, params if hp.wd_coupled != 0 else [], send, [send_off[j] for j in live],
                        [0] * len(live), [0] * len(live), [tasks[j].local_param.shape[1] for j in live], [], [],
                        hp.mode, hp.nesterov, hp.momentum,
                        hp.wd_coupled, part)
            sumsq.index_copy_(0, _h2d(live, torch.int64, send.device), part)

    def _cuda_owner_ns(self, tasks, hp, mine, shapes, rows_of, cnt, world, recv, shard_at, back, back_at,
                       parts) -> None:
        from .._ext import ext
        from ..ops.ns_cuda import round_up, run_ns_group, wide_shape

        E = ext()
        dev = recv.device
        # group owned matrices by their wide shape (tall ones transposed), so e.g. w1/w3 (14336x4096)
        # and w2 (4096x14336) of a SwiGLU FFN share one batched chain
        groups = _group_by(mine, lambda j: wide_shape(*shapes[j])[:2])
        for (mw, nw), js in groups.items():
            Mp, Np = round_up(mw), round_up(nw)
            per = 2 * Mp * Np * 2 + 2 * Mp * Mp * 2
            chunk = max(1, min(len(js), self.max_workspace_bytes // max(per, 1)))
            for c0 in range(0, len(js), chunk):
                sub = js[c0:c0 + chunk]
                tall_group = any(shapes[j][0] > shapes[j][1] for j in sub)
                B = len(sub)
                padded = (Mp != mw) or (Np != nw)
                X0 = (torch.zeros if padded else torch.empty)(B, Mp, Np, dtype=torch.bfloat16, device=dev)
                srcs, offs, row0, trs = [], [], [], []
                for b, j in enumerate(sub):
                    rws, cls = shapes[j]
                    tall = rws > cls
                    for r in range(world):
                        if rows_of[j][r] == 0:
                            continue
                        st = shard_at[(j, r)]
                        srcs.append(recv[st:st + cnt[j][r]].view(rows_of[j][r], cls))
                        offs.append(b * Mp * Np)
                        row0.append(chunk_offset(rws, world, r))
                        trs.append(int(tall))
                E.muon_prep(srcs, [], [], X0, offs, row0, trs, [Np], [], [], MODE_COPY, False, 0.0, 0.0, None)
                ssq = parts.index_select(1, _h2d(sub, torch.int64, dev)).contiguous()  # [world, B]
                s = torch.empty(B, dtype=torch.float32, device=dev)
                s2 = torch.empty_like(s)
                E.ns_scale(ssq, B, world, NS_EPS, s, s2)
                seg_views, meta = [], []
                for j in sub:
                    rws, cls = shapes[j]
                    cs = (rws + world - 1) // world
                    for d in range(world):
                        st = back_at[(j, d)]
                        # empty trailing shards still need a valid pointer
                        seg_views.append(back[st:st + max(cnt[j][d], 1)] if cnt[j][d] else back[:1])
                    meta += [cls, int(rws > cls), cs]
                ptrs = E.ptr_table(seg_views)
                meta_t = _h2d(meta, torch.int64, dev)
                run_ns_group(X0, s, s2, hp.ns_steps, ptrs, 0, False, False, mw, nw, p_scale=0.0, v_scale=1.0,
                             nseg=world, out_meta=meta_t, transposed_dest=tall_group)

    def _cuda_apply(self, tasks, ret, ret_at, cnt, rank) -> None:
        from .._ext import ext

        E = ext()
        idx = [j for j in range(len(tasks)) if tasks[j].local_param.numel() > 0]
        for key, js in _group_by(idx, lambda j: tasks[j].local_param.dtype).items():
            srcs = [ret[ret_at[j]:ret_at[j] + cnt[j][rank]].view(tasks[j].local_param.shape) for j in js]
            params = [tasks[j].local_param for j in js]
            E.muon_prep(srcs, [], params, None, [], [], [], [0], [_decay_float(tasks[j].decay) for j in js],
                        [-tasks[j].lr_eff for j in js], MODE_COPY, False, 0.0, 0.0, None)


# ---------------------------------------------------------------------- helpers
def _gather_list(x: torch.Tensor, world: int, group) -> List[torch.Tensor]:
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return parts


def _group_by(items, key) -> "OrderedDict":
    out: "OrderedDict" = OrderedDict()
    for it in items:
        out.setdefault(key(it), []).append(it)
    return out


def _momentum_torch(t: MuonTask, hp: MuonHyper) -> torch.Tensor:
    """Reference momentum math (optimizer.py:142-150 / fsdp.py:330-341) on the local shard."""
    g = t.local_grad
    if hp.wd_coupled != 0:
        g = g + hp.wd_coupled * t.local_param
    if hp.mode == MODE_COPY:
        return g
    buf = t.buf
    gb = g.to(buf.dtype)
    if hp.mode == MODE_EMA:
        buf.lerp_(gb, 1 - hp.momentum)
    else:
        buf.mul_(hp.momentum).add_(gb)
    if hp.nesterov:
        return gb + hp.momentum * buf
    return buf.clone()


def _decay_(p: torch.Tensor, decay) -> None:
    if isinstance(decay, torch.Tensor):
        p.mul_(decay.to(p.dtype))
    elif decay != 1.0:
        p.mul_(decay)


def _h2d(values, dtype, dev) -> torch.Tensor:
    """A small host-built tensor (pointer tables, indices, per-matrix scalars) on the device
    without a host synchronisation: staged in pinned memory, so the copy is asynchronous.  From
    pageable memory the copy waits for the stream's earlier work, which drains the queue and
    leaves the GPU idle while the host prepares the next launches."""
    t = torch.tensor(values, dtype=dtype)
    if torch.device(dev).type != "cuda":
        return t.to(dev)
    return t.pin_memory().to(dev, non_blocking=True)


def _decay_float(decay) -> float:
    return float(decay.item()) if isinstance(decay, torch.Tensor) else float(decay)


def _decay_vec(decays, dev) -> torch.Tensor:
    if all(not isinstance(d, torch.Tensor) for d in decays):
        return _h2d([float(d) for d in decays], torch.float32, dev)
    return torch.stack([torch.as_tensor(d, dtype=torch.float32, device=dev).reshape(()) for d in decays])
