"""Capacity reading of a recurrent memory: the delta rule's residual ratio
|v - S^T k| / |v| (``GDNLM.surprise``) averaged over sequences as a function
of position.  frac@p = share of the curve's total fall completed by position
p (comparable across geometries); plateau = the tail level (comparable only at
equal d_v).  Items are per (layer, bucket) means in a fixed order.

Parity: reference ``infra/eval/tasks/saturation.py:47-121``.
"""

from __future__ import annotations

from typing import Any, Sequence

import numpy as np
import torch

from ..core import EvalCtx, TaskResult

DEFAULT_EDGES = (1, 2, 4, 8, 16, 32, 64, 128, 192, 256, 384, 512, 1024)
DEFAULT_MARKS = (64, 128, 192, 256, 384, 512)


def _windows(store, rng, n: int, length: int) -> np.ndarray:
    w = np.asarray(store.shard_tokens, dtype=np.float64)
    w /= w.sum()
    out = []
    for _ in range(n):
        s = int(rng.choice(len(w), p=w))
        hi = int(store.shard_tokens[s]) - length - 1
        out.append(store.read_window(s, int(rng.integers(0, hi)), length))
    return np.stack(out).astype(np.int64)


def run(ctx: EvalCtx, data_dir: str, shards: list[str] | None = None, n_seqs: int = 32, length: int = 2048,
        batch_size: int = 8, edges: Sequence[int] = DEFAULT_EDGES, marks: Sequence[int] = DEFAULT_MARKS,
        tail_from: int = 1024) -> TaskResult:
    model: Any = ctx.subject.model
    assert hasattr(model, "surprise"), f"{type(model).__name__} has no surprise(); needs an all-GDN linear model"
    store = ctx.store(data_dir, shards)
    ids = _windows(store, ctx.rng("windows"), n_seqs, length)
    assert tail_from < length, f"tail_from {tail_from} must be inside length {length}"
    n_layers = int(model.config["layer_count"])
    acc = np.zeros((n_layers, length))
    seen = 0
    with torch.no_grad():
        for b in range(0, n_seqs, batch_size):
            tok = torch.from_numpy(ids[b:b + batch_size]).to(ctx.device)
            s = model.surprise(tok).mean(dim=(0, 3)).permute(1, 0).float().cpu().numpy()
            acc += s * tok.shape[0]
            seen += tok.shape[0]
    curve = acc / seen
    mean = curve.mean(0)
    lo_hi = [(lo, hi) for lo, hi in zip(edges[:-1], edges[1:]) if hi <= length]
    lo_hi.append((edges[-1], length))
    buckets = {f"b{lo}_{hi}": float(mean[lo:hi].mean()) for lo, hi in lo_hi}
    start, plateau = float(mean[0]), float(mean[tail_from:].mean())
    total = start - plateau
    fracs = {}
    if total > 0:
        for p in marks:
            if p < length:
                fracs[f"frac@{p}"] = float((start - mean[max(1, p - 8):p + 8].mean()) / total)
    scalars = {"start": start, "plateau": plateau, "total_fall": total,
               "fall_to_128": float(start - mean[120:136].mean()),
               "fall_after_128": float(mean[120:136].mean() - plateau), **fracs, **buckets}
    args = model.config
    return TaskResult(
        scalars=scalars,
        items={"bucket_mean": [float(curve[l, lo:hi].mean()) for l in range(n_layers) for lo, hi in lo_hi]},
        witness={"n_seqs": seen, "length": length, "tail_from": tail_from, "edges": list(edges), "marks": list(marks),
                 "buckets": [f"{lo}-{hi - 1}" for lo, hi in lo_hi],
                 "geometry": {k: args[k] for k in ("head_count", "key_head_dim", "value_head_dim")},
                 "rank_bound_d_k": int(args["key_head_dim"]),
                 "per_layer_plateau": [float(curve[l, tail_from:].mean()) for l in range(n_layers)],
                 "level_comparable_only_at_equal_d_v": int(args["value_head_dim"])})
