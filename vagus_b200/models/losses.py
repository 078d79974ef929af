"""Cross-entropy through the LM head, with an optional z-loss term.

Three implementations, numerically interchangeable at bf16 rounding:

* ``full``     logits materialised, then ``F.cross_entropy`` (largest peak).
* ``chunked``  rows processed in chunks under activation checkpointing; only
               one chunk of logits is ever alive.  Dependency-free oracle.
* ``fused``    the sm_100a fused linear cross-entropy
               (``vagus_b200.ops.fused_linear_ce``): per row chunk, the head
               GEMM writes bf16 logits, one kernel turns them into the loss,
               the log-sum-exp (for z-loss) and d(logits) in place, and two
               GEMMs produce d(hidden) and accumulate d(head weight) in fp32.
               ``liger`` is accepted as an alias (recipe compatibility).

``CELoss`` returns the combined objective (CE + z term); when z-loss is on,
``last_z`` holds the detached z term of the last call, so CE = loss - last_z.

Parity: reference ``infra/components/losses.py:1-138``.
"""

from __future__ import annotations

import torch
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from .. import ops

CE_IMPLS = ("full", "chunked", "fused", "liger")


def _chunk_sums(h, weight, targets, z_coef):
    logits = ops.linear(h, weight).float()
    ce = F.cross_entropy(logits, targets, reduction="sum")
    z = z_coef * torch.logsumexp(logits, dim=-1).pow(2).sum() if z_coef else logits.new_zeros(())
    return ce, z


def chunked_cross_entropy(hidden, weight, targets, *, chunk_rows: int = 4096, z_loss: float = 0.0,
                          return_z: bool = False):
    """Mean CE (+ z-loss) from hidden states without the full logits matrix."""
    h = hidden.reshape(-1, hidden.shape[-1])
    t = targets.reshape(-1)
    n = h.shape[0]
    ce_tot = torch.zeros((), device=h.device, dtype=torch.float32)
    z_tot = torch.zeros((), device=h.device, dtype=torch.float32)
    for i in range(0, n, chunk_rows):
        ce, z = checkpoint(_chunk_sums, h[i:i + chunk_rows], weight, t[i:i + chunk_rows], z_loss,
                           use_reentrant=False)
        ce_tot = ce_tot + ce
        z_tot = z_tot + z
    loss = (ce_tot + z_tot) / n
    return (loss, z_tot / n) if return_z else loss


class CELoss:
    """Callable ``(hidden, head_weight, targets) -> loss`` with z-term tracking."""

    def __init__(self, fn, tracks_z: bool):
        self._fn = fn
        self.tracks_z = tracks_z
        self.last_z: torch.Tensor | None = None

    def __call__(self, hidden, weight, targets) -> torch.Tensor:
        loss, z = self._fn(hidden, weight, targets)
        if z is not None:
            self.last_z = z
        return loss


def make_ce(impl: str, *, z_loss: float = 0.0, chunk_rows: int = 4096,
            compute_dtype: torch.dtype | None = torch.bfloat16) -> CELoss:
    if impl == "full":
        def full_fn(hidden, weight, targets):
            logits = ops.linear(hidden, weight)
            flat = logits.reshape(-1, logits.shape[-1])
            loss = F.cross_entropy(flat.float(), targets.reshape(-1))
            if not z_loss:
                return loss, None
            z = z_loss * torch.logsumexp(flat.float(), dim=-1).pow(2).mean()
            return loss + z, z.detach()
        return CELoss(full_fn, tracks_z=bool(z_loss))
    if impl == "chunked":
        def chunked_fn(hidden, weight, targets):
            loss, z = chunked_cross_entropy(hidden, weight, targets, chunk_rows=chunk_rows, z_loss=z_loss,
                                            return_z=True)
            return loss, (z.detach() if z_loss else None)
        return CELoss(chunked_fn, tracks_z=bool(z_loss))
    if impl in ("fused", "liger"):
        def fused_fn(hidden, weight, targets):
            if not hidden.is_cuda:
                loss, z = chunked_cross_entropy(hidden, weight, targets, chunk_rows=chunk_rows,
                                                z_loss=z_loss, return_z=True)
                return loss, (z.detach() if z_loss else None)
            loss, z = ops.fused_linear_ce(hidden.reshape(-1, hidden.shape[-1]), weight, targets.reshape(-1),
                                          z_loss=z_loss)
            return loss, (z.detach() if z_loss else None)
        return CELoss(fused_fn, tracks_z=bool(z_loss))
    raise KeyError(f"unknown fused ce impl '{impl}'")
