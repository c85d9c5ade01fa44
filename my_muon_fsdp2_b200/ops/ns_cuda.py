"""GPU orchestration of the batched Newton–Schulz chain (sm_100a kernels in ``csrc``).

A *group* is a set of matrices with the same (rows, cols).  The group is stacked into a
zero-padded bf16 workspace ``X0[B, Mp, Np]`` in the *wide* orientation (rows <= cols, the
tall ones transposed on the fly by the prep kernel), so that every GEMM of the chain is one
batched launch over the whole group:

    C1   A  = s^2 * X X^T            (symmetric, upper tiles + mirror; s^2 only on iteration 0)
    C2   B  = c * A A + b * A        (symmetric)
    C3   X' = s * (B X) + a * s * X  (B operand read MN-major from row-major X; s only on it. 0)

``s = 1 / (||G||_F + 1e-7)`` is folded into the epilogues, so the normalised X is never
materialised.  The last C3 writes straight into the destination tensors (pointer table) with
``T = p_scale * T + v_scale * X_final`` — for the Muon optimizer this is the parameter update
``p = (1 - lr*wd) * p - lr * scale * O`` (reference ``src/muon_fsdp/optimizer.py:157-170``).
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .._ext import ext
from .newton_schulz import NS_COEFFICIENTS, NS_EPS

PAD = 256  # every workspace dim is padded to the GEMM tile granularity


def round_up(x: int, m: int = PAD) -> int:
    return (x + m - 1) // m * m


def wide_shape(rows: int, cols: int) -> Tuple[int, int, bool]:
    """(rows_w, cols_w, transposed) of the wide orientation of a rows x cols matrix."""
    if rows > cols:
        return cols, rows, True
    return rows, cols, False


def run_ns_group(
    X0: torch.Tensor,
    s: torch.Tensor,
    s2: torch.Tensor,
    steps: int,
    out_ptrs: torch.Tensor,
    out_ld: int,
    out_f32: bool,
    out_transposed: bool,
    m_true: int,
    n_true: int,
    p_scale: float = 0.0,
    v_scale: float = 1.0,
    p_scale_vec: Optional[torch.Tensor] = None,
    v_scale_vec: Optional[torch.Tensor] = None,
    workspace: Optional[Dict[str, torch.Tensor]] = None,
    nseg: int = 1,
    out_meta: Optional[torch.Tensor] = None,
    transposed_dest: Optional[bool] = None,
) -> None:
    """Run ``steps`` quintic iterations on the stacked workspace and write the result out.

    ``X0`` is consumed (used as ping-pong storage).  ``workspace`` may provide reusable
    ``A``, ``B`` ([batch, Mp, Mp]) and ``X1`` ([batch, Mp, Np]) buffers.  ``out_ptrs`` holds
    ``batch * nseg`` destination pointers; with ``nseg > 1`` each destination row block of
    ``seg_rows`` rows (from ``out_meta``, int64 [batch, 3] = ld, transposed, seg_rows) goes to
    its own pointer (the scatter of each rank's row shard).

    ``transposed_dest`` (default ``out_transposed``) says whether the destinations hold the
    transpose of the workspace (tall matrices).  Then the last iteration writes the workspace
    and a tiled transpose kernel applies it: a GEMM epilogue that updates a transposed
    destination touches a different destination row for every element.
    """
    E = ext()
    a, b, c = NS_COEFFICIENTS
    batch, Mp, Np = X0.shape
    if steps == 0:
        E.ws_to_out(X0, s, out_ptrs, nseg, out_meta, out_ld, out_f32, out_transposed, m_true, n_true,
                    p_scale_vec, p_scale, v_scale_vec, v_scale)
        return
    ws = workspace or {}
    A = ws.get("A")
    if A is None or A.shape != (batch, Mp, Mp):
        A = torch.empty(batch, Mp, Mp, dtype=torch.bfloat16, device=X0.device)
    Bm = ws.get("B")
    if Bm is None or Bm.shape != (batch, Mp, Mp):
        Bm = torch.empty_like(A)
    if transposed_dest is None:
        transposed_dest = out_transposed
    X1 = ws.get("X1")
    if (steps > 1 or transposed_dest) and (X1 is None or X1.shape != X0.shape):
        X1 = torch.empty_like(X0)
    X = X0
    for it in range(steps):
        first = it == 0
        E.tc_gemm_ws(X, X, False, A, None, s2 if first else None, 1.0, None, 0.0, True)
        E.tc_gemm_ws(A, A, False, Bm, A, None, c, None, b, True)
        if it == steps - 1 and transposed_dest:
            E.tc_gemm_ws(Bm, X, True, X1, X, s if first else None, 1.0, s if first else None, a, False)
            E.ws_to_out(X1, None, out_ptrs, nseg, out_meta, out_ld, out_f32, out_transposed, m_true, n_true,
                        p_scale_vec, p_scale, v_scale_vec, v_scale)
        elif it == steps - 1:
            E.tc_gemm_out(Bm, X, True, X, s if first else None, 1.0, s if first else None, a, out_ptrs, nseg,
                          out_meta, out_ld, out_f32, out_transposed, m_true, n_true, p_scale_vec, p_scale,
                          v_scale_vec, v_scale)
        else:
            E.tc_gemm_ws(Bm, X, True, X1, X, s if first else None, 1.0, s if first else None, a, False)
            X, X1 = X1, X


def _as_supported(t: torch.Tensor) -> torch.Tensor:
    if t.dtype in (torch.float32, torch.bfloat16):
        return t.contiguous()
    return t.to(torch.float32).contiguous()


def newton_schulz_batched(
    mats: Sequence[torch.Tensor], steps: int = 5, out_dtype: Optional[torch.dtype] = None
) -> List[torch.Tensor]:
    """Orthogonalise CUDA matrices (any mix of shapes); one batched chain per shape group."""
    E = ext()
    results: List[Optional[torch.Tensor]] = [None] * len(mats)
    groups: "OrderedDict[Tuple[int, int, torch.dtype], List[int]]" = OrderedDict()
    for i, g in enumerate(mats):
        if g.dim() != 2:
            raise ValueError("newton_schulz_batched expects 2-D matrices")
        groups.setdefault((g.size(0), g.size(1), g.dtype), []).append(i)
    for (rows, cols, dtype), idxs in groups.items():
        dev = mats[idxs[0]].device
        mw, nw, tall = wide_shape(rows, cols)
        Mp, Np = round_up(mw), round_up(nw)
        B = len(idxs)
        X0 = torch.zeros(B, Mp, Np, dtype=torch.bfloat16, device=dev)
        sumsq = torch.zeros(B, dtype=torch.float32, device=dev)
        srcs = [_as_supported(mats[i]) for i in idxs]
        if len({t.dtype for t in srcs}) != 1:
            srcs = [t.float() for t in srcs]
        E.muon_prep(srcs, [], [], X0, [b * Mp * Np for b in range(B)], [0] * B, [int(tall)] * B, [Np], [], [], 0,
                    False, 0.0, 0.0, sumsq)
        s = torch.empty(B, dtype=torch.float32, device=dev)
        s2 = torch.empty_like(s)
        E.ns_scale(sumsq, B, 1, NS_EPS, s, s2)
        want = out_dtype or dtype
        store_dtype = want if want in (torch.float32, torch.bfloat16) else torch.float32
        outs = [torch.empty(rows, cols, dtype=store_dtype, device=dev) for _ in idxs]
        ptrs = E.ptr_table(outs)
        run_ns_group(X0, s, s2, steps, ptrs, cols, store_dtype == torch.float32, tall, mw, nw)
        for k, i in enumerate(idxs):
            results[i] = outs[k] if store_dtype == want else outs[k].to(want)
    return results  # type: ignore[return-value]
