"""RMSNorm with the statistics in at least fp32.

Parameter name ``gamma`` (checkpoint FQN compatibility).  On CUDA the forward
and backward are one fused sm_100a kernel each (``vagus_b200.ops.rmsnorm``);
on CPU the plain expression below is the oracle.

Parity: reference ``infra/components/norm_layer.py:4-24``.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import ops


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        assert dim > 0 and eps > 0
        self.dim = dim
        self.eps = eps
        self.gamma = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """``out_dtype`` lets a caller that feeds a bf16 GEMM ask for the bf16
        result directly (the fused kernel writes it without an fp32 copy)."""
        return ops.rmsnorm(x, self.gamma, self.eps, out_dtype=out_dtype)

    def extra_repr(self) -> str:
        return f"{self.dim}, eps={self.eps}"
