"""Linear layers on the tcgen05 GEMM.

Forward ``y = x W^T`` reads x (bf16, K-contiguous) and the bf16 compute copy
of W (K-contiguous); backward computes ``dx = dy W`` (W read N-contiguous, no
transpose) and ``dW = dy^T x`` straight into an fp32 gradient with the
split-K atomic epilogue.  ``linear_residual`` folds the residual add into the
GEMM epilogue: the kernel reads the fp32 residual and writes residual + x W^T.
"""

from __future__ import annotations

import torch
from torch.nn import functional as F

from ._core import BF16, as_bf16_2d, autocast_bf16, gemm


def gemm_ok(T: int, K: int, N: int) -> bool:
    """Shapes the tcgen05 GEMM takes in all three directions of a linear
    layer: every TMA box fits inside its tensor and rows are 16-byte pitched."""
    return T >= 128 and K >= 64 and N >= 128 and K % 8 == 0 and N % 8 == 0


def _wgrad(dy2: torch.Tensor, x2: torch.Tensor, shape) -> torch.Tensor:
    """fp32 dW (N x K) = dy^T (T x N)^T @ x (T x K), split-K atomics."""
    dW = torch.zeros(shape, device=dy2.device, dtype=torch.float32)
    gemm(dy2, True, x2, True, dW, atomic=True)
    return dW


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        x2 = as_bf16_2d(x)
        w16 = BF16.get(w)
        y = torch.empty(x2.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
        gemm(x2, False, w16, False, y)
        ctx.save_for_backward(x2, w)
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = as_bf16_2d(dy)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(x2.shape, device=x2.device, dtype=torch.bfloat16)
            gemm(dy2, False, BF16.get(w), True, dx)
            dx = dx.view(ctx.in_shape)
        if ctx.needs_input_grad[1]:
            dw = _wgrad(dy2, x2, w.shape)
        return dx, dw


class _LinearResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, resid, x, w):
        x2 = as_bf16_2d(x)
        r2 = resid.reshape(-1, resid.shape[-1])
        if r2.dtype != torch.float32 or not r2.is_contiguous():
            r2 = r2.float().contiguous()
        out = torch.empty_like(r2)
        gemm(x2, False, BF16.get(w), False, out, S=r2, beta=1.0)
        ctx.save_for_backward(x2, w)
        ctx.in_shape = x.shape
        return out.view(resid.shape)

    @staticmethod
    def backward(ctx, dout):
        x2, w = ctx.saved_tensors
        # the norm backward downstream may already have written a bf16 copy
        shadow = getattr(dout, "_vagus_bf16", None)
        if shadow is not None and shadow[1] == dout._version and shadow[0].shape == dout.shape:
            dy2 = shadow[0].view(-1, dout.shape[-1])
        else:
            dy2 = as_bf16_2d(dout)
        dx = dw = None
        if ctx.needs_input_grad[1]:
            dx = torch.empty(x2.shape, device=x2.device, dtype=torch.bfloat16)
            gemm(dy2, False, BF16.get(w), True, dx)
            dx = dx.view(ctx.in_shape)
        if ctx.needs_input_grad[2]:
            dw = _wgrad(dy2, x2, w.shape)
        return dout, dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` (no bias).  CPU: F.linear (the oracle, autocast applies).
    CUDA: the tcgen05 GEMM in bf16 whenever the input is bf16 or bf16
    autocast is on; an fp32 input outside autocast keeps fp32 arithmetic."""
    if not x.is_cuda:
        return F.linear(x, w)
    if x.dtype == torch.float32 and w.dtype == torch.float32 and not autocast_bf16():
        return F.linear(x, w)
    if x.numel() == 0 or not gemm_ok(x.numel() // x.shape[-1], x.shape[-1], w.shape[0]):
        # skinny shapes (gate projections, tiny test models): plain bf16 matmul
        return F.linear(x.to(torch.bfloat16), w.to(torch.bfloat16))
    return _Linear.apply(x, w)


def linear_residual(resid: torch.Tensor, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``resid + x @ w.T`` with the add fused into the GEMM epilogue (fp32 out)."""
    if not x.is_cuda or not gemm_ok(x.numel() // x.shape[-1], x.shape[-1], w.shape[0]):
        return resid + linear(x, w)
    return _LinearResidual.apply(resid, x, w)
