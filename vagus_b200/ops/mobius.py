"""Mobius-map scan x_t = (A_t x_{t-1} + B_t) / (C_t x_{t-1} + D_t) on CUDA
(``csrc/mobius.cu``: segment-composed 2x2 maps, then an exact fp32 replay of
the recurrence; the backward runs the adjoint recurrence the same way).

Parity: reference ``infra/components/kalman_delta.py:79-128``.
"""

from __future__ import annotations

import torch

from ._core import native


class _Mobius(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B, C, D, x0):
        X = native().mobius_fwd(A, B, C, D, x0)
        ctx.save_for_backward(A, B, C, D, x0, X)
        return X

    @staticmethod
    def backward(ctx, gX):
        gA, gB, gC, gD, gx0 = native().mobius_bwd(*ctx.saved_tensors, gX)
        return gA, gB, gC, gD, gx0


def mobius_scan(A, B, C, D, x0):
    """A..D: (batch, L, *rest) fp32 CUDA; x0: (batch, *rest).  Returns x
    (batch, L, *rest)."""
    b, L = A.shape[0], A.shape[1]
    rest = A.shape[2:]
    flat = lambda t: t.float().reshape(b, L, -1).contiguous()   # noqa: E731
    x = _Mobius.apply(flat(A), flat(B), flat(C), flat(D), x0.float().reshape(b, -1).contiguous())
    return x.view(b, L, *rest)
