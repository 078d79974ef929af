"""How sharp is each softmax-attention head, and which factor drives it?

With qk-norm both q and k are RMS-normalised per head, so a logit is
    q.k / sqrt(Dh) = sqrt(Dh) * rms(gamma_q) * rms(gamma_k) * cos(q, k)
up to the gammas' alignment with the vectors; ``ceiling`` = sqrt(Dh) *
|gamma_q|_inf * |gamma_k|_inf bounds every logit of the layer, and
observed max / ceiling is how far the heads' alignment goes.  A growing
ceiling (the 1-D gammas carry no weight decay) and growing cosines are
different problems; this separates them (``scale`` is the RMS form).

Per head on real tokens (materialised fp32 scores, causal):
  max logit   the largest pre-softmax logit
  gap         mean over query rows of top-1 minus top-2 logit (~20 nats:
              the row is one-hot and the head's pattern gets no gradient)
  entropy     mean row entropy (nats) and its ratio to the uniform ceiling
              log(i + 1)
  sink        mean attention mass on position 0
and, with a sigmoid output gate, its mean and the fractions above 0.9 and
below 0.1.

    python -m vagus_b200.meter.examples.probe_attention_health --ckpt A=runs/a/model-final.pt --data data/tok

Parity: reference ``infra/meter/examples/probe_attention_health.py``.
"""

from __future__ import annotations

import math

import torch

from ... import ops
from ._cli import probe_args, run_probe
from ._common import mixers, walk


@torch.no_grad()
def head_stats(att, h) -> dict:
    """Per-head sharpness of one softmax-attention module on input h."""
    B, L = h.shape[0], h.shape[1]
    qp, kp = ops.linear(h, att.wq.weight), ops.linear(h, att.wk.weight)
    if att.short_conv_size is not None:
        qp, kp = att.conv_q(qp), att.conv_k(kp)
    q, k = att._qk(qp, kp, 0)
    H, Dh = att.head_count, att.head_dim
    if att.kv_head_count != H:
        k = k.repeat_interleave(H // att.kv_head_count, dim=1)
    causal = torch.ones(L, L, dtype=torch.bool, device=h.device).tril()
    uni = torch.log(torch.arange(1, L + 1, device=h.device, dtype=torch.float32))
    out = {k_: [] for k_ in ("max_logit", "gap", "entropy", "entropy_ratio", "sink")}
    for hd in range(H):                                       # one head at a time: (B, L, L) fp32
        s = (q[:, hd].float() @ k[:, hd].float().transpose(-1, -2)) / math.sqrt(Dh)
        s = s.masked_fill(~causal, float("-inf"))
        p = s.softmax(-1)
        top = s.topk(2, dim=-1).values[:, 1:]                 # rows with at least two keys
        ent = -(p * p.clamp(min=1e-30).log()).sum(-1)         # (B, L)
        out["max_logit"].append(float(s.amax()))
        out["gap"].append(float((top[..., 0] - top[..., 1]).mean()) if L > 1 else 0.0)
        out["entropy"].append(float(ent.mean()))
        out["entropy_ratio"].append(float((ent[:, 1:] / uni[1:]).mean()) if L > 1 else 1.0)
        out["sink"].append(float(p[..., 0].mean()))
    if att.qk_norm:
        gq, gk = att.q_norm.gamma.float(), att.k_norm.gamma.float()
        out["ceiling"] = math.sqrt(Dh) * float(gq.abs().max() * gk.abs().max())
        out["scale"] = math.sqrt(Dh) * float(gq.pow(2).mean().sqrt() * gk.pow(2).mean().sqrt())
        out["max_cos"] = max(out["max_logit"]) / out["ceiling"] if out["ceiling"] > 0 else 0.0
    if att.out_gate:
        gate = torch.sigmoid(ops.linear(h, att.wg.weight).float())
        out["gate_mean"] = float(gate.mean())
        out["gate_open"] = float((gate > 0.9).float().mean())
        out["gate_shut"] = float((gate < 0.1).float().mean())
    return out


@torch.no_grad()
def probe(model, batches) -> dict:
    layers: dict[int, list[dict]] = {}
    for tokens in batches:
        def visit(i, blk, h):
            sm, _ = mixers(blk.att)
            if sm is not None:
                layers.setdefault(i, []).append(head_stats(sm, h))
        walk(model, tokens, visit)
    if not layers:
        raise ValueError("probe_attention_health: the model has no softmax-attention layer")
    report = {}
    for i, runs in sorted(layers.items()):
        merged = {}
        for key in runs[0]:
            vals = [r[key] for r in runs]
            if isinstance(vals[0], list):
                agg = max if key == "max_logit" else (lambda xs: sum(xs) / len(xs))
                merged[key] = [agg(col) for col in zip(*vals)]
            else:
                merged[key] = max(vals) if key in ("ceiling", "max_cos") else sum(vals) / len(vals)
        report[f"layer{i}"] = merged
    report["attn_logit_max"] = max(max(r["max_logit"]) for r in report.values() if isinstance(r, dict))
    return report


def render(r: dict) -> str:
    lines = [f"  attn_logit_max {r['attn_logit_max']:.2f}"]
    for name, s in r.items():
        if not isinstance(s, dict):
            continue
        head = f"  {name}:"
        if "ceiling" in s:
            head += f" ceiling {s['ceiling']:.1f} (rms scale {s['scale']:.1f})  max cos {s['max_cos']:.3f}"
        if "gate_mean" in s:
            head += f"  gate mean {s['gate_mean']:.2f} open {s['gate_open']:.2f} shut {s['gate_shut']:.2f}"
        lines.append(head)
        for hd in range(len(s["gap"])):
            lines.append(f"    head {hd:2d}: max {s['max_logit'][hd]:6.2f}  gap {s['gap'][hd]:6.2f}  "
                         f"entropy {s['entropy'][hd]:5.2f} ({100 * s['entropy_ratio'][hd]:3.0f}% of uniform)  "
                         f"sink {s['sink'][hd]:.3f}")
    return "\n".join(lines)


def main(argv=None):
    a = probe_args(__doc__).parse_args(argv)
    return run_probe(a, probe, render)


if __name__ == "__main__":
    main()
