"""Autograd wrappers of the transformer kernels (``csrc/model_kernels.cu``).

CUDA bf16 tensors run the sm_100a kernels; CPU tensors (and the reference checks in tests) run
plain PyTorch with the same math.  Every forward saves only what its backward needs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._ext import ext


def _cuda_bf16(*ts) -> bool:
    return all(t is not None and t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


# ---------------------------------------------------------------------------------- RMSNorm
class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        xc = x.contiguous()
        y, rstd = ext().rmsnorm_fwd(xc, w.contiguous(), eps)
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = ext().rmsnorm_bwd(dy.contiguous(), x, w.contiguous(), rstd)
        return dx, dw, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """y = x / sqrt(mean(x^2) + eps) * weight over the last dim."""
    if _cuda_bf16(x, weight):
        return _RMSNormFn.apply(x, weight, eps)
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * weight


# -------------------------------------------------------------------------------- LayerNorm
class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        xc = x.contiguous()
        y, mean, rstd = ext().layernorm_fwd(xc, w.contiguous(), None if b is None else b.contiguous(), eps)
        ctx.has_bias = b is not None
        ctx.save_for_backward(xc, w, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mean, rstd = ctx.saved_tensors
        dx, dw, db = ext().layernorm_bwd(dy.contiguous(), x, w.contiguous(), mean, rstd, ctx.has_bias)
        return dx, dw, (db if ctx.has_bias else None), None


def layer_norm(x, weight, bias=None, eps: float = 1e-5):
    if _cuda_bf16(x, weight) and (bias is None or _cuda_bf16(bias)):
        return _LayerNormFn.apply(x, weight, bias, eps)
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


# -------------------------------------------------------------------------------- embedding
class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, weight):
        ctx.save_for_backward(tokens)
        ctx.vocab = weight.shape[0]
        return ext().embedding_fwd(weight, tokens)

    @staticmethod
    def backward(ctx, dy):
        (tokens,) = ctx.saved_tensors
        if not ctx.needs_input_grad[1]:
            return None, None
        return None, ext().embedding_bwd(dy.contiguous(), tokens, ctx.vocab)


def embedding(tokens: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``weight[tokens]`` (an ``nn.Embedding`` lookup without padding_idx / max_norm); CUDA bf16
    tables run this library's gather and its one-pass dense backward."""
    if _cuda_bf16(weight) and tokens.is_cuda and weight.shape[1] % 8 == 0:
        return _EmbeddingFn.apply(tokens.long(), weight)
    return F.embedding(tokens, weight)


# ------------------------------------------------------------------------------------- RoPE
def _rope_torch(x: torch.Tensor, seq_len: int, theta: float, inverse: bool = False) -> torch.Tensor:
    """x: [B, T, H, D]; rotate-half convention (pairs (i, i + D/2))."""
    D = x.shape[-1]
    half = D // 2
    inv_freq = theta ** (-torch.arange(0, half, dtype=torch.float32, device=x.device) * 2.0 / D)
    pos = torch.arange(x.shape[1], dtype=torch.float32, device=x.device) % seq_len
    ang = pos[:, None] * inv_freq[None, :]
    cos, sin = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]
    if inverse:
        sin = -sin
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


class _RoPEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, theta):
        # x: [B, T, H, D] contiguous; rotated in place
        B, T, H, D = x.shape
        ext().rope_(x, B * T, H, D, T, theta, False, H * D, D)
        ctx.mark_dirty(x)
        ctx.theta = theta
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        B, T, H, D = g.shape
        ext().rope_(g, B * T, H, D, T, ctx.theta, True, H * D, D)
        return g, None


def apply_rope(x: torch.Tensor, theta: float = 10000.0) -> torch.Tensor:
    """Rotary embedding of x [B, T, H, D] at positions 0..T-1 (in place on CUDA)."""
    if _cuda_bf16(x) and x.is_contiguous():
        return _RoPEFn.apply(x, theta)
    return _rope_torch(x, x.shape[1], theta)


# ------------------------------------------------------------------------------ activations
class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        g, u = g.contiguous(), u.contiguous()
        ctx.save_for_backward(g, u)
        return ext().swiglu_fwd(g, u)

    @staticmethod
    def backward(ctx, d):
        g, u = ctx.saved_tensors
        dg, du = ext().swiglu_bwd(d.contiguous(), g, u)
        return dg, du


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up."""
    if _cuda_bf16(gate, up):
        return _SwiGLUFn.apply(gate, up)
    return F.silu(gate) * up


class _GELUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        ctx.save_for_backward(x)
        return ext().gelu_fwd(x)

    @staticmethod
    def backward(ctx, d):
        (x,) = ctx.saved_tensors
        return ext().gelu_bwd(d.contiguous(), x)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact (erf) GELU, like ``nn.GELU()``."""
    if _cuda_bf16(x):
        return _GELUFn.apply(x)
    return F.gelu(x)


# ----------------------------------------------------------------- LM head + cross entropy
class _LinearCEFn(torch.autograd.Function):
    """loss = mean_t CE(x_t @ W^T, y_t) with the logits computed chunk by chunk.

    Forward computes the gradients as well (the loss is terminal): per chunk the tcgen05 GEMM
    for the bf16 logits (``ops.linear``), the fused softmax-CE kernel that turns them into their
    gradient in place, then the tcgen05 GEMMs for dX (written into its row block) and dW (fp32
    accumulation across chunks, or bf16 for a single chunk).  Backward only scales by the
    incoming gradient.
    """

    @staticmethod
    def forward(ctx, x, w, targets, ignore_index, chunk):
        N, D = x.shape
        V = w.shape[0]
        valid = (targets != ignore_index).sum().clamp_min(1)
        dx = torch.empty_like(x)
        single = N <= chunk
        dw = None if single else torch.zeros(V, D, dtype=torch.float32, device=x.device)
        loss_sum = torch.zeros((), dtype=torch.float32, device=x.device)
        E = ext()
        inv = 1.0 / N  # kernel writes d(sum/N)/dlogits; rescaled by N/valid in backward
        from .linear import EPI_STORE, gemm, mm_dw, mm_fwd

        if single:
            dw = torch.empty(V, D, dtype=w.dtype, device=x.device)
        for s in range(0, N, chunk):
            e = min(N, s + chunk)
            xs = x[s:e]
            (logits,) = mm_fwd(xs, [w])  # [n, V] bf16
            rows = E.cross_entropy_(logits, targets[s:e].contiguous(), V, inv, ignore_index)
            loss_sum += rows.sum()
            gemm([logits], [w], False, True, [dx[s:e]], EPI_STORE)  # dX rows of this chunk
            mm_dw([logits], xs, [dw], accumulate=(s > 0))
        scale = N / valid.float()
        ctx.save_for_backward(dx, dw, scale)
        ctx.w_dtype = w.dtype
        return loss_sum / valid.float()

    @staticmethod
    def backward(ctx, g):
        dx, dw, scale = ctx.saved_tensors
        s = (g.float() * scale).reshape(1)  # stays on the device: no host synchronisation
        # the saved gradients are used once: scale them in place (one vectorised pass each)
        ext().scale_(dx, s)
        if dw.dtype == ctx.w_dtype:
            ext().scale_(dw, s)
        else:
            dw = (dw * s).to(ctx.w_dtype)
        return dx, dw, None, None, None


def fused_linear_cross_entropy(x: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                               ignore_index: int = -100, chunk: int = 8192) -> torch.Tensor:
    """Mean next-token CE of ``x @ weight.T`` against ``targets`` without materialising fp32 logits."""
    x2 = x.reshape(-1, x.shape[-1])
    t = targets.reshape(-1)
    if _cuda_bf16(x2, weight):
        return _LinearCEFn.apply(x2.contiguous(), weight, t, ignore_index, chunk)
    logits = (x2 @ weight.t()).float()
    return F.cross_entropy(logits, t, ignore_index=ignore_index)


# ---------------------------------------------------------------------------- attention
def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal attention with GQA. q: [B, T, Hq, D], k/v: [B, T, Hkv, D] -> [B, T, Hq, D]."""
    from .attention import flash_attention

    return flash_attention(q, k, v, causal=True)
