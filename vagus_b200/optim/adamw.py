"""AdamW whose CUDA step is one fused sm_100a kernel per parameter group
(flat fp32 views), with the exact update of ``torch.optim.AdamW``:

    m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
    p = p (1 - lr wd) - lr (m / bc1) / (sqrt(v / bc2) + eps)

On CPU it is ``torch.optim.AdamW`` itself.  The state dict layout (``step``,
``exp_avg``, ``exp_avg_sq`` per parameter) is torch's, so checkpoints move
between the two.
"""

from __future__ import annotations

import torch


class AdamW(torch.optim.AdamW):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, **kw):
        kw.pop("fused", None)
        kw.pop("foreach", None)
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, foreach=False, **kw)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        cuda_groups = [g for g in self.param_groups if any(p.is_cuda for p in g["params"])]
        if not cuda_groups:
            return super().step()
        from ..ops import native
        C = native()
        for g in self.param_groups:
            b1, b2 = g["betas"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                local = p.to_local() if hasattr(p, "to_local") else p
                grad = p.grad.to_local() if hasattr(p.grad, "to_local") else p.grad
                st = self.state[p]
                if not st:
                    st["step"] = torch.tensor(0.0)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                m = st["exp_avg"].to_local() if hasattr(st["exp_avg"], "to_local") else st["exp_avg"]
                v = st["exp_avg_sq"].to_local() if hasattr(st["exp_avg_sq"], "to_local") else st["exp_avg_sq"]
                if not local.is_cuda or local.dtype != torch.float32 or not local.is_contiguous():
                    raise RuntimeError("fused AdamW expects contiguous fp32 CUDA parameters")
                C.adamw_step(local.view(-1), grad.contiguous().view(-1).float(), m.view(-1), v.view(-1), None,
                             float(g["lr"]), float(b1), float(b2), float(g["eps"]), float(g["weight_decay"]),
                             int(st["step"].item()), 1.0)
        return loss
