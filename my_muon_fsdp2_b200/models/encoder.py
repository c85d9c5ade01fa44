"""Small models of the reference examples: the TransformerEncoder model
(``examples/fsdp_distributed.py:74-120``) and the MLP used by the CPU/gloo workload."""
from __future__ import annotations

import torch
import torch.nn as nn


class SimpleTransformer(nn.Module):
    """Embedding/projection + ``nn.TransformerEncoder`` (post-LN) + Linear head.

    ``input_dim`` switches the input from token ids (``vocab_size``) to dense features, which is
    the regression workload (inputs ~N(0,1), MSE to N(0,1) targets).
    """

    def __init__(self, vocab_size: int = 10000, d_model: int = 512, nhead: int = 8, num_layers: int = 6,
                 dim_feedforward: int = 2048, dropout: float = 0.0, input_dim: int = 0, output_dim: int = 0):
        super().__init__()
        self.input_dim = input_dim
        self.embed = nn.Linear(input_dim, d_model) if input_dim else nn.Embedding(vocab_size, d_model)
        layer = nn.TransformerEncoderLayer(d_model, nhead, dim_feedforward, dropout, batch_first=True)
        self.encoder = nn.TransformerEncoder(layer, num_layers, enable_nested_tensor=False)
        self.head = nn.Linear(d_model, output_dim or (input_dim or vocab_size))

    def forward(self, x):
        return self.head(self.encoder(self.embed(x)))

    def apply_fsdp2(self, mesh=None):
        """fully_shard every encoder layer, then the root."""
        from torch.distributed.fsdp import fully_shard

        for lyr in self.encoder.layers:
            fully_shard(lyr, mesh=mesh)
        fully_shard(self, mesh=mesh)
        return self


def mlp_512_2048_512(seed: int = 0) -> nn.Sequential:
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(512, 2048), nn.GELU(), nn.Linear(2048, 512))
