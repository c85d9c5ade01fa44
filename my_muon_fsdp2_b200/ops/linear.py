"""Transformer linears on this library's grouped tcgen05 GEMM (``csrc/linear_gemm.cu``).

The reference runs every projection as ``nn.Linear`` under ``fully_shard`` (library GEMMs;
examples/train_gpt.py:182-199 for the GPT-2 block).  Here each linear of a block, in all three
GEMMs of a training step (forward, input gradient, weight gradient), is one launch of the
grouped kernel, with the elementwise neighbours fused into its epilogue:

* ``qkv_rope``        q | k | v in one launch (three column segments), RoPE applied to q and k
                      in the epilogue; backward: one input-gradient launch over the three
                      reduction segments, one weight-gradient launch over the three row segments.
* ``swiglu_ffn``      W2 silu(W1 x) (W3 x) + residual: the two CTAs of each pair stage W1 and W3
                      rows of the same hidden units, so gate and up meet in TMEM and the epilogue
                      writes h = silu(g) u; W2's forward adds the residual in its epilogue; its
                      input-gradient GEMM applies the SwiGLU derivative in the epilogue, so dh is
                      never stored; dX = [dg du] [W1; W3] is one launch.
* ``linear``          y = x W^T (+ bias) (+ residual), e.g. the attention output projection.
* ``gelu_mlp``        GPT-2 MLP: W2 gelu(W1 x + b1) + b2 + residual, GELU and its derivative in
                      the epilogues.

Weights come either from plain parameters (also FSDP2-unsharded ones: their gradients flow back
through autograd) or from a ``SymmFSDP`` controller (``parallel/symm_fsdp.py``), which provides
the resident full weights and takes the weight gradients itself (partial sums straight into its
reduce-scatter buffers).  CPU tensors and other dtypes run the same math with PyTorch ops (the
oracle of the GPU tests).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .._ext import ext

EPI_STORE, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, EPI_GELU, EPI_GELU_BWD = range(6)


def _on_gpu(*ts) -> bool:
    return all(t is not None and t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


def gemm(A: Sequence[torch.Tensor], B: Sequence[torch.Tensor], a_mn: bool, b_mn: bool,
         out: Sequence[torch.Tensor], epilogue: int = EPI_STORE, C=None, aux0=None, aux1=None, bias=None,
         alpha: float = 1.0, accumulate: bool = False, rope_mask: int = 0, seq_len: int = 1, head_dim: int = 128,
         rope_theta: float = 0.0) -> None:
    """One launch of the grouped GEMM (argument layout: ``linear_gemm`` in csrc/bindings.cpp)."""
    ext().linear_gemm(list(A), list(B), a_mn, b_mn, list(out), epilogue, C, aux0, aux1, bias, float(alpha),
                      bool(accumulate), int(rope_mask), int(seq_len), int(head_dim), float(rope_theta))


def mm_fwd(x2: torch.Tensor, ws: Sequence[torch.Tensor], bias=None, residual=None) -> List[torch.Tensor]:
    """[x2 @ w^T for w in ws] in one launch (+ bias, + residual for a single weight)."""
    outs = [torch.empty(x2.shape[0], w.shape[0], dtype=x2.dtype, device=x2.device) for w in ws]
    gemm([x2], ws, False, False, outs, EPI_STORE, C=residual, bias=bias)
    return outs


def mm_dx(dys: Sequence[torch.Tensor], ws: Sequence[torch.Tensor], add_to: Optional[torch.Tensor] = None):
    """sum_s dys[s] @ ws[s] in one launch; with ``add_to`` the sum is added to it in place."""
    if add_to is not None:
        gemm(dys, ws, False, True, [add_to], EPI_STORE, C=add_to)
        return add_to
    dx = torch.empty(dys[0].shape[0], ws[0].shape[1], dtype=dys[0].dtype, device=dys[0].device)
    gemm(dys, ws, False, True, [dx], EPI_STORE)
    return dx


def mm_dw(dys: Sequence[torch.Tensor], x2: torch.Tensor, outs: Sequence[torch.Tensor], accumulate: bool) -> None:
    """outs[s] (+)= dys[s]^T @ x2 in one launch (outs bf16 or fp32)."""
    gemm(dys, [x2], True, True, outs, EPI_STORE, accumulate=accumulate)


# ------------------------------------------------------------------------ weight sources
class _Source:
    """Where the weights of a group of linears live and where their gradients go.

    Plain weights: the tensors themselves; the weight gradients are returned through autograd.
    SymmFSDP linears: the controller's resident full weights (gathered by its fused all-gather
    GEMM on the first forward of a step); the controller accumulates the gradients itself.
    """

    def __init__(self, mods):
        ctl = getattr(mods[0], "_symm_ctl", None)
        self.ctl = ctl if ctl is not None and all(getattr(m, "_symm_ctl", None) is ctl for m in mods) else None
        self.idxs = tuple(m._symm_idx for m in mods) if self.ctl is not None else ()

    def needs_gather(self) -> bool:
        return self.ctl is not None and not self.ctl.resident(self.idxs)

    def weights(self, tensors=()) -> List[torch.Tensor]:
        """Full weights: the controller's resident copies, or the given plain tensors."""
        if self.ctl is not None:
            return [self.ctl.full_weight(i) for i in self.idxs]
        return list(tensors)

    def saved(self, ws) -> Tuple[torch.Tensor, ...]:
        """What a function saves for its backward: the plain weights (none for the controller)."""
        return () if self.ctl is not None else tuple(ws)

    def plain_forward(self, x2) -> List[torch.Tensor]:
        """The products through the controller's own forward (fused all-gather GEMM)."""
        return [self.ctl.linear_forward(i, x2) for i in self.idxs]

    def weight_grads(self, dys, x2, need, sel: Optional[Sequence[int]] = None) -> Tuple[Optional[torch.Tensor], ...]:
        """Gradients of the weights at positions ``sel`` of this source (default: all) from their
        output gradients ``dys`` and the shared input ``x2``."""
        if self.ctl is not None:
            sel = range(len(self.idxs)) if sel is None else sel
            self.ctl.accumulate_grads([self.idxs[k] for k in sel], list(dys), x2)
            return (None,) * len(dys)
        if not any(need):
            return (None,) * len(dys)
        outs = [torch.empty(d.shape[1], x2.shape[1], dtype=d.dtype, device=d.device) for d in dys]
        mm_dw(dys, x2, outs, accumulate=False)
        return tuple(o if n else None for o, n in zip(outs, need))


def _rope_(t: torch.Tensor, T: int, heads: int, hd: int, theta: float, inverse: bool) -> None:
    ext().rope_(t, t.shape[0], heads, hd, T, theta, inverse, heads * hd, hd)


# ---------------------------------------------------------------------------- q | k | v
class _QKVRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, src, T, hd, theta, *ws):
        if src.needs_gather():
            q, k, v = src.plain_forward(x2)
            _rope_(q, T, q.shape[1] // hd, hd, theta, False)
            _rope_(k, T, k.shape[1] // hd, hd, theta, False)
        else:
            W = src.weights(ws)
            q, k, v = [torch.empty(x2.shape[0], w.shape[0], dtype=x2.dtype, device=x2.device) for w in W]
            gemm([x2], W, False, False, [q, k, v], EPI_ROPE, rope_mask=0b011, seq_len=T, head_dim=hd,
                 rope_theta=theta)
        ctx.save_for_backward(x2, *src.saved(ws))
        ctx.src, ctx.T, ctx.hd, ctx.theta = src, T, hd, theta
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2, *ws = ctx.saved_tensors
        src, T, hd, theta = ctx.src, ctx.T, ctx.hd, ctx.theta
        dq, dk, dv = dq.contiguous().clone(), dk.contiguous().clone(), dv.contiguous()
        _rope_(dq, T, dq.shape[1] // hd, hd, theta, True)
        _rope_(dk, T, dk.shape[1] // hd, hd, theta, True)
        W = src.weights(ws)
        dx = mm_dx([dq, dk, dv], W) if ctx.needs_input_grad[0] else None
        gw = src.weight_grads([dq, dk, dv], x2, ctx.needs_input_grad[5:8])
        return (dx, None, None, None, None) + gw


def _rope_torch(x: torch.Tensor, T: int, hd: int, theta: float) -> torch.Tensor:
    from .model_ops import _rope_torch as rt

    M, N = x.shape
    return rt(x.view(M // T, T, N // hd, hd), T, theta).reshape(M, N)


def qkv_rope(x: torch.Tensor, mods, seq_len: int, head_dim: int, theta: float):
    """(rope(x Wq^T), rope(x Wk^T), x Wv^T) for x [..., D] with T = seq_len consecutive tokens per
    sequence; 2-D results [tokens, heads * head_dim]."""
    x2 = x.reshape(-1, x.shape[-1])
    src = _Source(mods)
    W = [m.weight for m in mods]
    if _on_gpu(x2) and head_dim in (64, 128) and (src.ctl is not None or _on_gpu(*W)):
        return _QKVRopeFn.apply(x2.contiguous(), src, seq_len, head_dim, theta, *W)
    if src.ctl is not None:
        from ..parallel.symm_fsdp import multi_linear

        q, k, v = multi_linear(x2, mods)
    else:
        q, k, v = (F.linear(x2, w) for w in W)
    return _rope_torch(q, seq_len, head_dim, theta), _rope_torch(k, seq_len, head_dim, theta), v


# ---------------------------------------------------------------------- SwiGLU FFN
class _SwiGLUFFNFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, residual, src, *ws):
        M = x2.shape[0]
        if src.needs_gather():
            # first forward of the step on several ranks: the fused all-gather GEMMs gather
            # W1, W3 and W2 (products unfused with SwiGLU this once)
            g, u = [src.ctl.linear_forward(i, x2) for i in src.idxs[:2]]
            h = ext().swiglu_fwd(g, u)
            y = src.ctl.linear_forward(src.idxs[2], h)
            if residual is not None:
                y.add_(residual)
        else:
            W1, W3, W2 = src.weights(ws)
            F_ = W1.shape[0]
            h, g, u = (torch.empty(M, F_, dtype=x2.dtype, device=x2.device) for _ in range(3))
            gemm([x2], [W1, W3], False, False, [h, g, u], EPI_SWIGLU)
            y = torch.empty(M, W2.shape[0], dtype=x2.dtype, device=x2.device)
            gemm([h], [W2], False, False, [y], EPI_STORE, C=residual)
        ctx.save_for_backward(x2, h, g, u, *src.saved(ws))
        ctx.src = src
        ctx.has_res = residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, h, g, u, *ws = ctx.saved_tensors
        src = ctx.src
        dy = dy.contiguous()
        W1, W3, W2 = src.weights(ws)
        dg, du = torch.empty_like(g), torch.empty_like(u)
        # dH = dY W2 never leaves the tensor memory: the epilogue writes dg and du
        gemm([dy], [W2], False, True, [dg, du], EPI_SWIGLU_BWD, aux0=g, aux1=u)
        need = ctx.needs_input_grad
        gw2 = src.weight_grads([dy], h, need[5:6], sel=(2,))
        dx = mm_dx([dg, du], [W1, W3]) if need[0] else None
        gw13 = src.weight_grads([dg, du], x2, need[3:5], sel=(0, 1))
        return (dx, dy if ctx.has_res else None, None) + gw13 + gw2


def swiglu_ffn(x: torch.Tensor, w1, w3, w2, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """w2(silu(w1(x)) * w3(x)) (+ residual), modules w1, w3, w2 (weights [F, D], [F, D], [D, F])."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    src = _Source((w1, w3, w2))
    W = [w1.weight, w3.weight, w2.weight]
    if _on_gpu(x2) and (src.ctl is not None or _on_gpu(*W)) and (r2 is None or _on_gpu(r2)):
        y = _SwiGLUFFNFn.apply(x2.contiguous(), None if r2 is None else r2.contiguous(), src, *W)
        return y.view(*shape[:-1], y.shape[-1])
    from .model_ops import swiglu

    if src.ctl is not None:
        from ..parallel.symm_fsdp import multi_linear

        g, u = multi_linear(x2, (w1, w3))
        y = w2(swiglu(g, u))
    else:
        y = F.linear(swiglu(F.linear(x2, W[0]), F.linear(x2, W[1])), W[2])
    y = y.view(*shape[:-1], y.shape[-1])
    return y if residual is None else y + residual


# -------------------------------------------------------------------- single linear
class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, residual, bias, src, w):
        if src.needs_gather():
            (y,) = src.plain_forward(x2)
            if bias is not None:
                y.add_(bias)
            if residual is not None:
                y.add_(residual)
        else:
            (W,) = src.weights([w])
            (y,) = mm_fwd(x2, [W], bias=bias, residual=residual)
        ctx.save_for_backward(x2, *src.saved([w]))
        ctx.src, ctx.has_res, ctx.has_bias = src, residual is not None, bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, *ws = ctx.saved_tensors
        src = ctx.src
        dy = dy.contiguous()
        (W,) = src.weights(ws)
        need = ctx.needs_input_grad
        dx = mm_dx([dy], [W]) if need[0] else None
        db = dy.sum(0) if ctx.has_bias and need[2] else None
        (gw,) = src.weight_grads([dy], x2, need[4:5])
        return dx, (dy if ctx.has_res else None), db, None, gw


def linear(x: torch.Tensor, mod, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mod(x) (+ residual) with the residual added in the GEMM epilogue."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    src = _Source((mod,))
    b = getattr(mod, "bias", None)
    if _on_gpu(x2) and (src.ctl is not None or _on_gpu(mod.weight)) and (r2 is None or _on_gpu(r2)) and \
            (b is None or _on_gpu(b)):
        y = _LinearFn.apply(x2.contiguous(), None if r2 is None else r2.contiguous(), b, src, mod.weight)
        return y.view(*shape[:-1], y.shape[-1])
    y = mod(x)
    return y if residual is None else y + residual


# ---------------------------------------------------------------------- GELU MLP (GPT-2)
class _GeluMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, residual, b1, b2, src, w1, w2):
        M = x2.shape[0]
        W1, W2 = src.weights([w1, w2])
        a = torch.empty(M, W1.shape[0], dtype=x2.dtype, device=x2.device)
        z = torch.empty_like(a)
        gemm([x2], [W1], False, False, [a, z], EPI_GELU, bias=b1)
        (y,) = mm_fwd(a, [W2], bias=b2, residual=residual)
        ctx.save_for_backward(x2, a, z, *src.saved([w1, w2]))
        ctx.src, ctx.has_res = src, residual is not None
        ctx.has_b1, ctx.has_b2 = b1 is not None, b2 is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, a, z, *ws = ctx.saved_tensors
        src = ctx.src
        dy = dy.contiguous()
        W1, W2 = src.weights(ws)
        need = ctx.needs_input_grad
        dz = torch.empty_like(z)
        gemm([dy], [W2], False, True, [dz], EPI_GELU_BWD, aux0=z)
        db2 = dy.sum(0) if ctx.has_b2 and need[3] else None
        db1 = dz.sum(0) if ctx.has_b1 and need[2] else None
        (gw2,) = src.weight_grads([dy], a, need[6:7], sel=(1,))
        dx = mm_dx([dz], [W1]) if need[0] else None
        (gw1,) = src.weight_grads([dz], x2, need[5:6], sel=(0,))
        return dx, (dy if ctx.has_res else None), db1, db2, None, gw1, gw2


def gelu_mlp(x: torch.Tensor, fc, proj, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """proj(gelu(fc(x))) (+ residual), exact-erf GELU (as ``nn.GELU()``)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    src = _Source((fc, proj))
    b1, b2 = getattr(fc, "bias", None), getattr(proj, "bias", None)
    ok = _on_gpu(x2) and src.ctl is None and _on_gpu(fc.weight, proj.weight) and (r2 is None or _on_gpu(r2)) and \
        (b1 is None or _on_gpu(b1)) and (b2 is None or _on_gpu(b2))
    if ok:
        y = _GeluMLPFn.apply(x2.contiguous(), None if r2 is None else r2.contiguous(), b1, b2, src, fc.weight,
                             proj.weight)
        return y.view(*shape[:-1], y.shape[-1])
    from .model_ops import gelu

    y = proj(gelu(fc(x)))
    return y if residual is None else y + residual
