"""Where does a delta-rule memory stop learning about the stream?

The per-token residual rho_t = |v_t - S_{t-1}^T k_t| / |v_t| (from a blank
state) is what the memory failed to predict about the value it is about to
store.  It falls while the d_k x d_v state fills and flattens once the keys
stop being separable (about d_k tokens), so the position of the knee is a
structural read of the memory's capacity that needs no task the model can
solve.  The recurrence is ``GatedDeltaNet.residuals`` (fp32 token loop, the
same decay / read / residual / write steps as the layer's own scan).

Reports per model: rho at geometric positions, the plateau (mean over the
last quarter of the window), the knee (first position within 5% of the
plateau, measured from rho at position 0) and the share of the total drop
reached by position d_k.

    python -m vagus_b200.meter.examples.saturation_curve \\
        --ckpt A=runs/a/ckpt-00005000.pt --ckpt B=runs/b/ckpt-00005000.pt --data data/tok --batches 4

Parity: reference ``infra/meter/examples/saturation_curve.py``.
"""

from __future__ import annotations

import torch

from ._cli import probe_args, run_probe
from ._common import mixers, walk


@torch.no_grad()
def probe(model, batches) -> dict:
    curves, dk = [], None
    for tokens in batches:
        per_layer = []

        def visit(i, blk, h):
            nonlocal dk
            _, la = mixers(blk.att)
            if la is not None and la.delta:
                per_layer.append(la.residuals(h).mean(dim=(0, 2)))        # (L,)
                dk = la.key_head_dim
        walk(model, tokens, visit)
        if not per_layer:
            raise ValueError("saturation_curve: the model has no delta-rule layer")
        curves.append(torch.stack(per_layer))                              # (layers, L)
    rho = torch.stack(curves).mean(0)                                      # (layers, L)
    return summarise(rho, dk)


def summarise(rho: torch.Tensor, dk: int) -> dict:
    """rho (layers, L) -> the report (model-wide mean curve plus per layer)."""
    L = rho.shape[1]
    mean = rho.mean(0)

    def read(c):
        plateau = float(c[-max(1, L // 4):].mean())
        start = float(c[0])
        drop = start - plateau
        knee = L
        if drop > 0:
            hit = (c <= plateau + 0.05 * drop).nonzero()
            knee = int(hit[0]) + 1 if len(hit) else L
        at_dk = float(c[min(dk, L) - 1])
        learned = (start - at_dk) / drop if drop > 0 else 1.0
        return {"rho_start": start, "plateau": plateau, "knee": knee, "learned_by_dk": learned}

    pos, p = [], 1
    while p <= L:
        pos.append(p)
        p *= 2
    if pos[-1] != L:
        pos.append(L)
    return {"key_dim": dk, "positions": pos, "rho": [float(mean[q - 1]) for q in pos], **read(mean),
            "layers": [read(rho[i]) for i in range(rho.shape[0])]}


def render(r: dict) -> str:
    lines = ["  position " + " ".join(f"{p:>6d}" for p in r["positions"]),
             "  rho      " + " ".join(f"{v:6.3f}" for v in r["rho"]),
             f"  plateau {r['plateau']:.3f}  knee at {r['knee']}  "
             f"{100 * r['learned_by_dk']:.0f}% of the drop by position d_k = {r['key_dim']}"]
    for i, lr in enumerate(r["layers"]):
        lines.append(f"  layer {i:2d}: start {lr['rho_start']:.3f} plateau {lr['plateau']:.3f} knee {lr['knee']}")
    return "\n".join(lines)


def main(argv=None):
    a = probe_args(__doc__).parse_args(argv)
    return run_probe(a, probe, render)


if __name__ == "__main__":
    main()
