"""How much of a stream a recurrent memory still absorbs, by position.

The delta rule writes beta k (v - S^T k)^T: the residual ratio
|v - S^T k| / |v| (``GDNLM.surprise``) is the part of the incoming value the
memory could not predict.  Averaged over sequences from a blank state it
falls while the state has room and levels off when it has not; where it
levels off is the memory's practical horizon, which the learned decay can
set well below the d_k rank bound.

Scalars: ``start`` (position 0), ``plateau`` (mean from ``tail_from`` on),
``total_fall`` = start - plateau, ``fall_to_128`` / ``fall_after_128``
(around positions 120..135, when the length covers them), ``frac@p`` for p in ``marks`` -- the share of
the total fall done by p (a 16-position average around p), emitted only when
the curve falls (an untrained model's rises) -- and ``b<lo>_<hi>`` bucket
means over ``edges``.  ``frac@p`` compares across geometries; levels only at
equal d_v (the ratio is relative to |v|).  Items: per (layer, bucket) means,
layer-major, for pairing; the per-layer plateaus are in the witness.

Windows: contiguous, token-weighted (``Draws.window`` with one token of
slack, salt ``"windows"``) -- the training distribution.

Parity: reference ``infra/eval/tasks/saturation.py`` (arguments, draws,
scalar and item definitions).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from ..core import EvalCtx, TaskResult

DEFAULT_EDGES = (1, 2, 4, 8, 16, 32, 64, 128, 192, 256, 384, 512, 1024)
DEFAULT_MARKS = (64, 128, 192, 256, 384, 512)


def _buckets(edges: Sequence[int], length: int) -> list[tuple[int, int]]:
    out = [(lo, hi) for lo, hi in zip(edges[:-1], edges[1:]) if hi <= length]
    return out + [(edges[-1], length)]


def run(ctx: EvalCtx, data_dir: str, shards: list[str] | None = None, n_seqs: int = 32, length: int = 2048,
        batch_size: int = 8, edges: Sequence[int] = DEFAULT_EDGES, marks: Sequence[int] = DEFAULT_MARKS,
        tail_from: int = 1024) -> TaskResult:
    model = ctx.subject.model
    if not hasattr(model, "surprise"):
        raise TypeError(f"saturation needs a model with surprise() (an all-GDN GDNLM), not {type(model).__name__}")
    if tail_from >= length:
        raise ValueError(f"saturation: tail_from {tail_from} must lie inside length {length}")
    store = ctx.store(data_dir, shards)
    draws = ctx.draws(store, "windows")
    ids = np.stack([draws.read(*draws.window(length, slack=1), length) for _ in range(n_seqs)])
    layers = int(model.config["layer_count"])
    curve = np.zeros((layers, length))
    with torch.no_grad():
        for b in range(0, n_seqs, batch_size):
            tok = torch.from_numpy(ids[b:b + batch_size]).to(ctx.device)
            r = model.surprise(tok)                            # (B, L, layers, H)
            curve += r.float().mean(dim=3).sum(dim=0).T.cpu().numpy()
            ctx.log(f"saturation: {min(b + batch_size, n_seqs)}/{n_seqs} sequences")
    curve /= n_seqs
    mean = curve.mean(0)
    spans = _buckets(edges, length)
    start, plateau = float(mean[0]), float(mean[tail_from:].mean())
    fall = start - plateau
    scalars = {"start": start, "plateau": plateau, "total_fall": fall}
    if length >= 136:                                  # the 120..135 window exists
        near128 = float(mean[120:136].mean())
        scalars.update(fall_to_128=start - near128, fall_after_128=near128 - plateau)
    if fall > 0:
        for p in marks:
            if p < length:
                scalars[f"frac@{p}"] = float((start - mean[max(1, p - 8):p + 8].mean()) / fall)
    scalars.update({f"b{lo}_{hi}": float(mean[lo:hi].mean()) for lo, hi in spans})
    cfg = model.config
    return TaskResult(
        scalars=scalars,
        items={"bucket_mean": [float(curve[l, lo:hi].mean()) for l in range(layers) for lo, hi in spans]},
        witness={"n_seqs": n_seqs, "length": length, "tail_from": tail_from, "edges": list(edges),
                 "marks": list(marks), "buckets": [f"{lo}-{hi - 1}" for lo, hi in spans],
                 "geometry": {k: cfg[k] for k in ("head_count", "key_head_dim", "value_head_dim")},
                 "rank_bound_d_k": int(cfg["key_head_dim"]),
                 "per_layer_plateau": [float(curve[l, tail_from:].mean()) for l in range(layers)],
                 "level_comparable_only_at_equal_d_v": int(cfg["value_head_dim"])})
