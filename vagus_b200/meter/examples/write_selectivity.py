"""Is the delta-rule write selective, or does every token cost the same?

The write S <- S + w_t r_t^T moves the state by |w_t| |r_t| (r_t the
residual; for the symmetric write w_t = beta_t k_t with unit keys, |w_t| is
beta_t).  A state with d_k slots under a stream of thousands of tokens is
oversubscribed, so what it spends its writes on is the question.  Three
reads per model, over every delta-rule layer, head and token:

  corr(w, rho)    Pearson correlation of |w| with the residual ratio rho,
                  per (layer, head), averaged: does the gate know what the
                  memory failed to predict?
  write gain      mean |w| on the 10% most surprising tokens over mean |w|
                  on the least surprising half (1.0: no selectivity).
  concentration   share of the total |w| * rho held by the top k% of tokens
                  (k% when uniform): selectivity from the gate and from the
                  residual together.

The write goes through the layer's own ``_write`` hook, so a Kalman mixer's
asymmetric write is measured as |w| of its write vector.

    python -m vagus_b200.meter.examples.write_selectivity --ckpt A=runs/a/model-final.pt --data data/tok

Parity: reference ``infra/meter/examples/write_selectivity.py``.
"""

from __future__ import annotations

import torch

from ... import ops
from ...models.scans import residual_scan
from ._cli import probe_args, run_probe
from ._common import mixers, walk

TOPS = (1, 5, 10, 25)


@torch.no_grad()
def layer_writes(la, h):
    """(|w|, rho), each (B, L, H) fp32, of one delta-rule layer on input h
    (None when the layer has no write strength)."""
    q, k, v = la._heads(ops.linear(h, la.wq.weight), ops.linear(h, la.wk.weight), ops.linear(h, la.wv.weight))
    g, beta = la._gates(h)
    beta, w = la._write(h, k, g, beta)
    if beta is None and w is None:
        return None
    rho = residual_scan(k, v, g, beta, None, delta=True, w=w)
    mag = w.float().norm(dim=-1) if w is not None else beta.float() * k.float().norm(dim=-1)
    return mag, rho


def _corr(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Pearson correlation along dim 0 (one value per remaining index)."""
    a = a - a.mean(0)
    b = b - b.mean(0)
    return (a * b).sum(0) / (a.norm(dim=0) * b.norm(dim=0)).clamp(min=1e-12)


@torch.no_grad()
def probe(model, batches) -> dict:
    per_layer: dict[int, list] = {}
    for tokens in batches:
        def visit(i, blk, h):
            _, la = mixers(blk.att)
            wr = layer_writes(la, h) if la is not None and la.delta else None
            if wr is not None:
                per_layer.setdefault(i, []).append(wr)
        walk(model, tokens, visit)
    if not per_layer:
        raise ValueError("write_selectivity: the model has no delta-rule layer with a write strength")
    mags, rhos, corrs = [], [], []
    for i, parts in sorted(per_layer.items()):
        m = torch.cat([p[0].reshape(-1, p[0].shape[-1]) for p in parts])    # (tokens, H)
        r = torch.cat([p[1].reshape(-1, p[1].shape[-1]) for p in parts])
        corrs.append(_corr(m, r))
        mags.append(m.flatten())
        rhos.append(r.flatten())
    m, r = torch.cat(mags), torch.cat(rhos)
    order = r.argsort(descending=True)
    n = len(r)
    top10, bottom = order[:max(1, n // 10)], order[n // 2:]
    gain = float(m[top10].mean() / m[bottom].mean().clamp(min=1e-12))
    mass = (m * r).sort(descending=True).values
    total = float(mass.sum())
    conc = {f"top{k}%": float(mass[:max(1, n * k // 100)].sum()) / total for k in TOPS}
    return {"tokens": n, "w_mean": float(m.mean()), "w_median": float(m.median()), "rho_mean": float(r.mean()),
            "corr_w_rho": float(torch.cat(corrs).mean()), "corr_per_layer": [float(c.mean()) for c in corrs],
            "write_gain": gain, "concentration": conc}


def render(r: dict) -> str:
    conc = "  ".join(f"{k} {100 * v:.1f}%" for k, v in r["concentration"].items())
    return (f"  |w| mean {r['w_mean']:.3f} median {r['w_median']:.3f}   rho mean {r['rho_mean']:.3f}   "
            f"({r['tokens']} token-heads)\n"
            f"  corr(|w|, rho) {r['corr_w_rho']:+.3f}   per layer "
            + " ".join(f"{c:+.2f}" for c in r["corr_per_layer"]) + "\n"
            f"  write gain {r['write_gain']:.3f}   concentration of |w|*rho: {conc}")


def main(argv=None):
    a = probe_args(__doc__).parse_args(argv)
    return run_probe(a, probe, render)


if __name__ == "__main__":
    main()
