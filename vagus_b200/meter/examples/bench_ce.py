"""Linear cross-entropy over the vocabulary: the fused kernel path
(``make_ce('fused')``, logits never materialised in full) against the plain
path (``make_ce('full')``) and, when it is installed, liger's fused linear
cross-entropy (the reference's default), forward+backward time and peak
memory, z-loss 1e-4 in all three.

    python -m vagus_b200.meter.examples.bench_ce --T 32768 --D 1024 --V 32000
"""

from __future__ import annotations

import argparse

import torch

from ...models.losses import make_ce
from ..compare import compare


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--T", type=int, default=32768, help="tokens")
    ap.add_argument("--D", type=int, default=1024)
    ap.add_argument("--V", type=int, default=32000)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    h = torch.randn(1, a.T, a.D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    w = (0.02 * torch.randn(a.V, a.D, device=dev)).to(torch.bfloat16).requires_grad_(True)
    y = torch.randint(0, a.V, (1, a.T), device=dev)
    variants = {}
    for impl in ("full", "fused"):
        ce = make_ce(impl, z_loss=1e-4)

        def run(ce=ce):
            loss = ce(h, w, y)
            return torch.autograd.grad(loss, (h, w))[0]
        variants[impl] = run
    if dev == "cuda":
        try:
            from liger_kernel.transformers.fused_linear_cross_entropy import LigerFusedLinearCrossEntropyLoss
        except ImportError:
            LigerFusedLinearCrossEntropyLoss = None
        if LigerFusedLinearCrossEntropyLoss is not None:
            lg = LigerFusedLinearCrossEntropyLoss(lse_square_scale=1e-4)

            def run_liger():
                loss = lg(w, h.view(-1, a.D), y.view(-1))
                return torch.autograd.grad(loss, (h, w))[0]
            variants["liger"] = run_liger
    compare(variants, ref="full", iters=a.iters)


if __name__ == "__main__":
    main()
