"""GPT-2 (pre-LN, learned positions, GELU MLP 4x, tied LM head).

Same architecture and configs as the reference example (``examples/train_gpt.py:49-268``:
small 768/12/12, medium 1024/24/16, large 1280/36/20, vocab 50257, ctx 1024), with the naive
O(T^2) masked attention replaced by causal flash attention, the linears on this library's
grouped tcgen05 GEMM (GELU, biases and residual adds in its epilogues), LayerNorm on its kernels
and the tied head fused with the cross entropy.  ``configure_fsdp`` shards every block
*and* the root (the reference leaves the root unsharded, train_gpt.py:265-268).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from ..ops.linear import gelu_mlp, linear
from ..ops.model_ops import causal_attention, embedding, fused_linear_cross_entropy, gelu, layer_norm


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    n_positions: int = 1024
    n_embd: int = 768
    n_layer: int = 12
    n_head: int = 12
    embd_pdrop: float = 0.0
    resid_pdrop: float = 0.0
    attn_pdrop: float = 0.0
    layer_norm_epsilon: float = 1e-5


def GPT2SmallConfig() -> GPTConfig:
    return GPTConfig()


def GPT2MediumConfig() -> GPTConfig:
    return GPTConfig(n_embd=1024, n_layer=24, n_head=16)


def GPT2LargeConfig() -> GPTConfig:
    return GPTConfig(n_embd=1280, n_layer=36, n_head=20)


class LayerNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        return layer_norm(x, self.weight, self.bias, self.eps)


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.n_head = cfg.n_head
        self.head_dim = cfg.n_embd // cfg.n_head
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd)
        self.resid_dropout = nn.Dropout(cfg.resid_pdrop)

    def forward(self, x, residual: Optional[torch.Tensor] = None):
        """c_proj(attention(c_attn(x))) (+ residual: added in c_proj's GEMM epilogue when the
        dropout between them is inactive)."""
        B, T, C = x.shape
        q, k, v = linear(x, self.c_attn).split(C, dim=2)
        q = q.reshape(B, T, self.n_head, self.head_dim)
        k = k.reshape(B, T, self.n_head, self.head_dim)
        v = v.reshape(B, T, self.n_head, self.head_dim)
        y = causal_attention(q, k, v).reshape(B, T, C)
        if self.training and self.resid_dropout.p > 0:
            y = self.resid_dropout(linear(y, self.c_proj))
            return y if residual is None else residual + y
        return linear(y, self.c_proj, residual)


class MLP(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.c_fc = nn.Linear(cfg.n_embd, 4 * cfg.n_embd)
        self.c_proj = nn.Linear(4 * cfg.n_embd, cfg.n_embd)
        self.dropout = nn.Dropout(cfg.resid_pdrop)

    def forward(self, x, residual: Optional[torch.Tensor] = None):
        """c_proj(gelu(c_fc(x))) (+ residual), GELU and its derivative in the GEMM epilogues."""
        if self.training and self.dropout.p > 0:
            y = self.dropout(self.c_proj(gelu(self.c_fc(x))))
            return y if residual is None else residual + y
        return gelu_mlp(x, self.c_fc, self.c_proj, residual)


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.ln_1 = LayerNorm(cfg.n_embd, cfg.layer_norm_epsilon)
        self.attn = CausalSelfAttention(cfg)
        self.ln_2 = LayerNorm(cfg.n_embd, cfg.layer_norm_epsilon)
        self.mlp = MLP(cfg)

    def forward(self, x):
        x = self.attn(self.ln_1(x), residual=x)
        return self.mlp(self.ln_2(x), residual=x)


class GPTModel(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.config = cfg
        self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.n_positions, cfg.n_embd)
        self.drop = nn.Dropout(cfg.embd_pdrop)
        self.h = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)])
        self.ln_f = LayerNorm(cfg.n_embd, cfg.layer_norm_epsilon)
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(m: nn.Module) -> None:
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, 0.0, 0.02)
            if getattr(m, "bias", None) is not None:
                nn.init.zeros_(m.bias)

    def forward(self, input_ids: torch.Tensor, targets: Optional[torch.Tensor] = None):
        B, T = input_ids.shape
        if T > self.config.n_positions:
            raise ValueError(f"Sequence length {T} exceeds maximum {self.config.n_positions}")
        pos = torch.arange(T, device=input_ids.device)
        x = self.drop(embedding(input_ids, self.wte.weight) + embedding(pos, self.wpe.weight))
        for blk in self.h:
            x = blk(x)
        x = self.ln_f(x)
        if targets is None:
            return x @ self.wte.weight.t()
        return fused_linear_cross_entropy(x, self.wte.weight, targets)

    def configure_fsdp(self, mesh=None) -> None:
        from torch.distributed.fsdp import fully_shard

        for blk in self.h:
            fully_shard(blk, mesh=mesh)
        fully_shard(self, mesh=mesh)

    def muon_param_names(self):
        return [n for n, p in self.named_parameters() if p.dim() == 2 and n.startswith("h.")]
