"""Teacher-forced statistics on windows of real text, one scoring pass, many
metrics (``LOGIT_METRICS``: fn(logp, targets, args) -> {name: (B,) tensor}).

Windows are sampled by seed from the store, read as L tokens and scored as
the stream start_id + window[:-1]; the start-token-only prediction is dropped.
Several lengths share the same window starts (nested prefixes); lengths above
a subject's ``max_stream_len`` are skipped and listed in the witness.

nll / ppl, entropy, top_p_support (nucleus size at top_p, the sampling rule),
rep_at_l (Welleck et al.: argmax prediction found among the previous l gold
tokens, the same for the gold token itself, and the excess).

Parity: reference ``infra/eval/tasks/holdout.py:42-138``.
"""

from __future__ import annotations

import math
from collections import defaultdict
from typing import Sequence

import numpy as np
import torch
import torch.nn.functional as F

from ..core import EvalCtx, TaskResult, exposure


def metric_nll(logp, targets, args):
    return {"nll": -logp.gather(-1, targets[..., None]).squeeze(-1).mean(1)}


def metric_entropy(logp, targets, args):
    return {"entropy": -(logp.exp() * logp).sum(-1).mean(1)}


def metric_top_p_support(logp, targets, args):
    p = logp.exp().sort(dim=-1, descending=True).values
    kept = ((p.cumsum(-1) - p) < args["top_p"]).sum(-1)
    return {"top_p_support": kept.float().mean(1)}


def metric_rep_at_l(logp, targets, args):
    pred = logp.argmax(-1)
    out = {}
    for l in args["rep_l"]:
        prev = F.pad(targets, (l, 0), value=-1).unfold(1, l, 1)[:, :-1]
        rep = (prev == pred[..., None]).any(-1).float().mean(1)
        gold = (prev == targets[..., None]).any(-1).float().mean(1)
        out[f"rep_{l}"], out[f"gold_rep_{l}"], out[f"rep_excess_{l}"] = rep, gold, rep - gold
    return out


LOGIT_METRICS = {"nll": metric_nll, "entropy": metric_entropy, "top_p_support": metric_top_p_support,
                 "rep_at_l": metric_rep_at_l}


def run(ctx: EvalCtx, data_dir: str, shards: list[str] | None = None, n_seq: int = 128,
        context_len: int | list[int] = 2048, batch_size: int = 4,
        metrics: Sequence[str] = ("nll", "entropy", "top_p_support", "rep_at_l"), top_p: float = 0.9,
        rep_l: Sequence[int] = (32, 128)) -> TaskResult:
    store = ctx.store(data_dir, shards)
    lengths = sorted({int(x) for x in ([context_len] if isinstance(context_len, int) else context_len)})
    L_max = lengths[-1]
    rng = ctx.rng("windows")
    w = np.asarray(store.shard_tokens, dtype=np.float64)
    w /= w.sum()
    windows = []
    for _ in range(n_seq):
        s = int(rng.choice(len(w), p=w))
        windows.append((s, int(rng.integers(0, store.shard_tokens[s] - L_max))))
    gen = ctx.subject.generator
    limit = gen.model.max_stream_len
    args = {"top_p": top_p, "rep_l": tuple(int(l) for l in rep_l)}
    result = TaskResult()
    ran, skipped = [], []
    for L in lengths:
        if limit is not None and L > limit:
            skipped.append(L)
            continue
        per: dict[str, list[float]] = defaultdict(list)
        for b0 in range(0, n_seq, batch_size):
            batch = windows[b0:b0 + batch_size]
            ids = torch.tensor(np.stack([store.read_window(s, st, L).astype(np.int64) for s, st in batch]))
            logits = gen.score_ids(ids)[:, 1:]
            targets = ids[:, 1:].to(logits.device)
            logp = logits.float().log_softmax(-1)
            del logits
            for name in metrics:
                for k, v in LOGIT_METRICS[name](logp, targets, args).items():
                    per[k].extend(v.float().cpu().tolist())
            del logp
        for k, v in per.items():
            result.items[f"{k}@{L}"] = v
            result.scalars[f"{k}@{L}"] = float(np.mean(v))
        if "nll" in per:
            result.scalars[f"ppl@{L}"] = math.exp(result.scalars[f"nll@{L}"])
        ran.append(L)
        ctx.log(f"  L={L}: " + " ".join(f'{k}={result.scalars[f"{k}@{L}"]:.4f}' for k in per))
    result.witness = {"n_seq": n_seq, "lengths": ran, "lengths_skipped": skipped, "metrics": list(metrics),
                      "top_p": top_p, "rep_l": list(args["rep_l"]),
                      "store": {"dir": str(store.dir.resolve()), "source": store.manifest.get("source"),
                                "tokenizer": store.manifest.get("tokenizer", {}).get("id"),
                                "shards": [e["file"] for e in store.entries], "total_tokens": store.total_tokens},
                      "exposure": exposure(ctx.subject, store),
                      "windows": [[store.entries[s]["file"], st] for s, st in windows]}
    return result
