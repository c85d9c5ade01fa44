"""Llama-3-style decoder (RMSNorm, RoPE theta=500000, GQA attention, SwiGLU FFN, untied LM head).

The reference has no Llama; this is the model of the Llama-3 8B FSDP2+Muon workload
(32 layers, d=4096, 32 query / 8 KV heads, head_dim 128, FFN 14336, vocab 128256).
Every projection runs on this library's grouped tcgen05 GEMM (``ops.linear``): q | k | v in one
launch with RoPE in its epilogue, W1 | W3 with SwiGLU in the epilogue, and the residual adds of
the attention output projection and of W2 fused into their GEMMs.  The embedding lookup, RMSNorm,
attention and the LM-head cross entropy are this library's sm_100a kernels as well
(``ops.model_ops``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from ..ops.linear import linear, qkv_rope, swiglu_ffn
from ..ops.model_ops import causal_attention, embedding, fused_linear_cross_entropy, rms_norm


@dataclass
class LlamaConfig:
    vocab_size: int = 128256
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    ffn_dim: int = 14336
    rope_theta: float = 500000.0
    norm_eps: float = 1e-5
    max_seq_len: int = 8192
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @classmethod
    def llama3_8b(cls) -> "LlamaConfig":
        return cls()

    @classmethod
    def tiny(cls, **kw) -> "LlamaConfig":
        base = dict(vocab_size=512, dim=128, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=256, max_seq_len=256)
        base.update(kw)
        return cls(**base)

    def num_params(self) -> int:
        d, f, hd = self.dim, self.ffn_dim, self.head_dim
        attn = d * (self.n_heads * hd) + 2 * d * (self.n_kv_heads * hd) + (self.n_heads * hd) * d
        layer = attn + 3 * d * f + 2 * d
        return self.n_layers * layer + 2 * self.vocab_size * d + d


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        hd = cfg.head_dim
        self.wq = nn.Linear(cfg.dim, cfg.n_heads * hd, bias=False)
        self.wk = nn.Linear(cfg.dim, cfg.n_kv_heads * hd, bias=False)
        self.wv = nn.Linear(cfg.dim, cfg.n_kv_heads * hd, bias=False)
        self.wo = nn.Linear(cfg.n_heads * hd, cfg.dim, bias=False)

    def forward(self, x, residual: Optional[torch.Tensor] = None):
        """wo(attention(rope(wq x), rope(wk x), wv x)) (+ residual, added in wo's epilogue)."""
        B, T, _ = x.shape
        c = self.cfg
        q, k, v = qkv_rope(x, (self.wq, self.wk, self.wv), T, c.head_dim, c.rope_theta)
        q = q.view(B, T, c.n_heads, c.head_dim)
        k = k.view(B, T, c.n_kv_heads, c.head_dim)
        v = v.view(B, T, c.n_kv_heads, c.head_dim)
        o = causal_attention(q, k, v)
        return linear(o.reshape(B, T, -1), self.wo, residual)


class FeedForward(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.w1 = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.w3 = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.w2 = nn.Linear(cfg.ffn_dim, cfg.dim, bias=False)

    def forward(self, x, residual: Optional[torch.Tensor] = None):
        """w2(silu(w1 x) * w3 x) (+ residual)."""
        return swiglu_ffn(x, self.w1, self.w3, self.w2, residual)


class TransformerBlock(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.attention_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.attention = Attention(cfg)
        self.ffn_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.feed_forward = FeedForward(cfg)

    def forward(self, x):
        h = self.attention(self.attention_norm(x), residual=x)
        return self.feed_forward(self.ffn_norm(h), residual=h)


class Llama(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.tok_embeddings = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.layers = nn.ModuleList([TransformerBlock(cfg) for _ in range(cfg.n_layers)])
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.output = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)

    @torch.no_grad()
    def init_weights(self, seed: int = 0) -> None:
        """N(0, init_std) for matrices, ones for norms; works on FSDP2 DTensor shards."""
        g = torch.Generator(device="cpu").manual_seed(seed)
        for name, p in self.named_parameters():
            local = p.to_local() if hasattr(p, "to_local") else p
            if name.endswith("norm.weight") or "norm." in name:
                local.fill_(1.0)
            else:
                # per-rank stream: different shards get different values
                gen = torch.Generator(device=local.device).manual_seed(seed * 1000003 + hash(name) % 1000003 +
                                                                       _rank_offset())
                local.normal_(0.0, self.cfg.init_std, generator=gen)

    def forward(self, tokens: torch.Tensor, targets: Optional[torch.Tensor] = None):
        x = embedding(tokens, self.tok_embeddings.weight)
        for layer in self.layers:
            x = layer(x)
        x = self.norm(x)
        if targets is None:
            return linear(x, self.output)
        return fused_linear_cross_entropy(x, self.output.weight, targets)

    def muon_param_names(self):
        """Attention and FFN matrices (Muon); everything else (embeddings, norms, LM head) -> AdamW."""
        return [n for n, p in self.named_parameters() if p.dim() == 2 and (".attention." in n or ".feed_forward." in n)]


def _rank_offset() -> int:
    import torch.distributed as dist

    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def apply_fsdp(model: nn.Module, mesh=None, reshard_after_forward: bool = True, blocks_attr: str = "layers"):
    """``fully_shard`` every block and then the root (FSDP2)."""
    from torch.distributed.fsdp import fully_shard

    for blk in getattr(model, blocks_attr):
        fully_shard(blk, mesh=mesh, reshard_after_forward=reshard_after_forward)
    fully_shard(model, mesh=mesh, reshard_after_forward=reshard_after_forward)
    return model
