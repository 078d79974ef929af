"""Rotary position embedding, interleaved-pair convention.

Pairs are channels (2i, 2i+1) of a head: ``y0 = x0 cos - x1 sin``,
``y1 = x0 sin + x1 cos`` with angle ``pos * base^(-i / (Dh/2))``.  The cos/sin
tables are built in fp32 and shared by every layer (one module per model);
``prepare_m(L)`` grows them.  The tables are non-persistent buffers.

Parity: reference ``infra/components/pos_embed.py:7-75``.
"""

from __future__ import annotations

import torch
from torch import nn


class RoPE(nn.Module):
    mcos: torch.Tensor
    msin: torch.Tensor

    def __init__(self, dim: int, head_dim: int, context_len: int, base: float = 10000.0):
        super().__init__()
        assert dim % head_dim == 0 and head_dim > 0 and head_dim % 2 == 0
        assert context_len > 0 and base > 1
        self.dim = dim
        self.head_dim = head_dim
        self.context_len = context_len
        self.base = base
        self.half = head_dim // 2
        self.prepared_L = 0
        self.register_buffer("mcos", torch.zeros(()), persistent=False)
        self.register_buffer("msin", torch.zeros(()), persistent=False)
        self.prepare_m(context_len)

    def prepare_m(self, L: int) -> None:
        if L <= self.prepared_L:
            return
        dev, dt = self.mcos.device, self.mcos.dtype
        inv = torch.pow(self.base, -torch.arange(self.half, device=dev, dtype=torch.float32) / self.half)
        ang = torch.arange(L, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.register_buffer("mcos", torch.cos(ang).to(dt), persistent=False)
        self.register_buffer("msin", torch.sin(ang).to(dt), persistent=False)
        self.prepared_L = L

    def tables(self, L: int, offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        if offset + L > self.prepared_L:
            raise ValueError("Context length exceeded. Please call RoPE.prepare_m to enlarge.")
        return self.mcos[offset:offset + L], self.msin[offset:offset + L]

    def forward(self, x: torch.Tensor, offset: int = 0) -> torch.Tensor:
        """x: (..., L, head_dim)."""
        assert x.shape[-1] == self.head_dim
        cos, sin = self.tables(x.shape[-2], offset)
        pairs = x.reshape(*x.shape[:-1], self.half, 2)
        x0, x1 = pairs[..., 0], pairs[..., 1]
        y = torch.stack((x0 * cos - x1 * sin, x0 * sin + x1 * cos), dim=-1)
        return y.reshape(x.shape)
