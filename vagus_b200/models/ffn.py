"""SwiGLU feed-forward: ``l2(silu(x1) * gate)`` with ``[x1; gate] = l1(x)``.

``l1.weight`` rows are ``[x1 rows; gate rows]`` (checkpoint layout).  Init is
Transformer++: N(0, init_std) on ``l1``, ``l2`` shrunk by 1/sqrt(2 L).

Parity: reference ``infra/components/ffn.py:7-52``.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .. import ops


class FFN(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, init_std: float = 0.02,
                 layer_count: int | None = None):
        super().__init__()
        assert dim > 0 and hidden_dim > 0
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.l1 = nn.Linear(dim, 2 * hidden_dim, bias=False)
        self.l2 = nn.Linear(hidden_dim, dim, bias=False)
        nn.init.normal_(self.l1.weight, std=init_std)
        nn.init.normal_(self.l2.weight, std=init_std / math.sqrt(2 * layer_count) if layer_count else init_std)

    def hidden(self, x: torch.Tensor) -> torch.Tensor:
        """The SwiGLU activation, the input of ``l2``."""
        return ops.swiglu(ops.linear(x, self.l1.weight))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(self.hidden(x), self.l2.weight)
