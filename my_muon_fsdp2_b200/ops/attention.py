"""Causal (GQA) attention entry point used by the model zoo.

``flash_attention(q, k, v, causal=True)`` with q [B, T, Hq, D] and k, v [B, T, Hkv, D].
CUDA: PyTorch's ``scaled_dot_product_attention`` (cuDNN / flash backends, a library kernel)
until the native sm_100a attention kernel lands; CPU: the same op in fp32-safe math.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True) -> torch.Tensor:
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    out = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, enable_gqa=(Hq != Hkv))
    return out.transpose(1, 2)
