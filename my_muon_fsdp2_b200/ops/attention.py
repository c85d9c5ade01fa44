"""Causal (GQA) flash attention: ``flash_attention(q, k, v, causal=True)``.

q: [B, T, Hq, D], k/v: [B, T, Hkv, D] -> [B, T, Hq, D].  CUDA bf16 inputs with D in {64, 128}
run the tcgen05 kernels of ``csrc/attention.cu`` (forward and backward; the forward saves the
row log-sum-exp for the backward).  T is padded up to a multiple of 128 internally: padded keys
sit after every real query and are masked by causality; padded queries are sliced off and
receive zero upstream gradient.  CPU tensors (and non-causal use) go through PyTorch's
``scaled_dot_product_attention``.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .._ext import ext
from ..utils.tracing import nvtx_range


def _pad_t(x: torch.Tensor, tp: int) -> torch.Tensor:
    if x.shape[1] == tp:
        return x.contiguous()
    return F.pad(x, (0, 0, 0, 0, 0, tp - x.shape[1])).contiguous()


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v):
        T = q.shape[1]
        tp = (T + 127) // 128 * 128
        qp, kp, vp = _pad_t(q, tp), _pad_t(k, tp), _pad_t(v, tp)
        scale = 1.0 / math.sqrt(q.shape[-1])
        with nvtx_range("attention/forward"):
            o, lse = ext().attention_fwd(qp, kp, vp, scale)
        ctx.save_for_backward(qp, kp, vp, o, lse)
        ctx.T, ctx.scale = T, scale
        return o[:, :T] if tp != T else o

    @staticmethod
    def backward(ctx, do):
        qp, kp, vp, o, lse = ctx.saved_tensors
        T = ctx.T
        dop = _pad_t(do, qp.shape[1])
        with nvtx_range("attention/backward"):
            dq, dk, dv = ext().attention_bwd(dop, qp, kp, vp, o, lse, ctx.scale)
        if qp.shape[1] != T:
            dq, dk, dv = dq[:, :T], dk[:, :T], dv[:, :T]
        return dq, dk, dv


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True) -> torch.Tensor:
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    if (causal and q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and D in (64, 128)
            and Hq % Hkv == 0):
        return _FlashAttnFn.apply(q, k, v)
    if q.is_cuda and q.dtype == torch.bfloat16 and causal:
        raise RuntimeError(f"flash_attention: unsupported CUDA shape (head_dim {D}, heads {Hq}/{Hkv})")
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    out = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, enable_gqa=(Hq != Hkv))
    return out.transpose(1, 2)
