"""Depthwise causal short convolution over the sequence (K taps).

One parameter, ``conv.weight`` of shape (D, 1, K) (an ``nn.Conv1d`` so the
checkpoint layout matches), one semantics: ``y[t] = sum_i w[:, K-1-i] x[t-i]``
with zeros before the start.  ``impl`` is accepted for recipe compatibility
('conv1d', 'shift', 'fla'); on CUDA the GatedDeltaNet layer never calls this
module's forward -- its fused sm_100a kernel does conv + SiLU (+ L2 norm) for
q, k and v in one launch -- so the choice only selects how the CPU oracle is
written.

Parity: reference ``infra/components/opt.py:15-93``.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

CONV_IMPLS = ("conv1d", "shift", "fla")


def _act(y: torch.Tensor, activation: str | None) -> torch.Tensor:
    if activation is None:
        return y
    assert activation in ("silu", "swish"), activation
    return F.silu(y)


class ShortConv(nn.Module):
    def __init__(self, dim: int, kernel: int, impl: str = "conv1d"):
        super().__init__()
        assert dim > 0 and kernel > 0
        assert impl in CONV_IMPLS, f"{impl!r} not in {CONV_IMPLS}"
        self.kernel = kernel
        self.impl = impl
        self.conv = nn.Conv1d(dim, dim, kernel, groups=dim, bias=False)

    def forward(self, x: torch.Tensor, activation: str | None = None) -> torch.Tensor:
        """(B, L, D) -> (B, L, D), causal."""
        if self.impl == "conv1d":
            # the weight in the activations' dtype (bf16 activations over fp32 master weights)
            y = F.conv1d(F.pad(x.transpose(1, 2), (self.kernel - 1, 0)), self.conv.weight.to(x.dtype),
                         groups=self.conv.groups).transpose(1, 2)
        else:
            y = self.shifted(x)
        return _act(y, activation)

    def shifted(self, x: torch.Tensor) -> torch.Tensor:
        """The same convolution as K shifted multiply-adds."""
        w = self.conv.weight[:, 0, :].to(x.dtype)          # (D, K)
        K = self.kernel
        y = x * w[:, K - 1]
        for i in range(1, K):
            if i >= x.shape[1]:
                break
            y = y + F.pad(x[:, :-i], (0, 0, i, 0)) * w[:, K - 1 - i]
        return y

    def direct_conv(self, x: torch.Tensor, activation: str | None = None) -> torch.Tensor:
        """Unpadded convolution (decode path): output length L - K + 1."""
        return _act(self.conv(x.transpose(1, 2)).transpose(1, 2), activation)
