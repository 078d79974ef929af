"""Fused linear cross-entropy (+ z-loss) on the tcgen05 GEMM.

Per row chunk: the head GEMM writes bf16 logits; one kernel per row computes
the log-sum-exp, the row loss and overwrites the logits with
d(loss)/d(logits); then d(hidden) = dlogits W and d(W) += dlogits^T hidden
(fp32, split-K atomics).  The gradients are produced during the forward (only
one chunk of logits is ever alive) and scaled by the incoming gradient in
backward.
"""

from __future__ import annotations

import torch

from ._core import BF16, as_bf16_2d, gemm, native

CHUNK_ROWS = 8192


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, targets, z_coef):
        h2 = as_bf16_2d(h)
        w16 = BF16.get(w)
        N, D = h2.shape
        V = w.shape[0]
        tg = targets.reshape(-1).to(torch.long).contiguous()
        scale = 1.0 / N
        dh = torch.empty(N, D, device=h.device, dtype=torch.bfloat16)
        dW = torch.zeros(V, D, device=h.device, dtype=torch.float32)
        rows = min(CHUNK_ROWS, N)
        logits = torch.empty(rows, V, device=h.device, dtype=torch.bfloat16)
        loss_sum = torch.zeros((), device=h.device, dtype=torch.float32)
        z_sum = torch.zeros((), device=h.device, dtype=torch.float32)
        C = native()
        for r0 in range(0, N, rows):
            r1 = min(N, r0 + rows)
            hc = h2[r0:r1]
            lg = logits[: r1 - r0]
            gemm(hc, False, w16, False, lg)
            lr, lse = C.softmax_ce(lg, tg[r0:r1], scale, z_coef)
            loss_sum += lr.sum()
            if z_coef:
                z_sum += lse.square().sum()
            gemm(lg, False, w16, True, dh[r0:r1])
            gemm(lg, True, hc, True, dW, atomic=True)
        z = z_sum * (z_coef / N)
        loss = loss_sum / N + z
        ctx.save_for_backward(dh, dW)
        ctx.mark_non_differentiable(z)
        ctx.h_shape = h.shape
        return loss, z

    @staticmethod
    def backward(ctx, gloss, gz):
        dh, dW = ctx.saved_tensors
        return (dh * gloss.to(dh.dtype)).view(ctx.h_shape), dW * gloss, None, None


def fused_linear_ce(hidden, weight, targets, z_loss: float = 0.0):
    """Mean CE of ``hidden @ weight.T`` against ``targets`` plus
    ``z_loss * mean(lse^2)``; returns (loss, z_term)."""
    return _FusedLinearCE.apply(hidden, weight, targets, float(z_loss or 0.0))
