"""Teacher-forced statistics of a subject on windows of real text: one
scoring pass per batch, every requested statistic from the same
log-probabilities.

Windows of the longest requested length are drawn by ``Draws.window``
(salt ``"windows"``); a shorter length scores the prefix of the same
windows, so lengths are nested.  Each window is scored as a stream (start
token + the window): L tokens, of which the L - 1 after the first are scored
with the context training gave them.  Lengths beyond the subject's
``max_stream_len`` are skipped and listed (how a NoPE or linear model's
extrapolation is read against a RoPE model's).

Statistics (per sequence, then averaged; ``<name>@<L>`` keys):

  nll            mean -log p(token)             (and ppl@L = exp(nll@L))
  entropy        mean predictive entropy, nats
  top_p_support  mean nucleus size at ``top_p`` (the tokens a top-p sampler
                 would choose among; the rule of ``inference.sampling``)
  rep_at_l       for l in ``rep_l``: rep_l, the share of positions whose
                 argmax occurs among the previous l text tokens; gold_rep_l,
                 the same for the true token (the text's own repetition);
                 rep_excess_l = rep_l - gold_rep_l  (Welleck et al., 2019)

Parity: reference ``infra/eval/tasks/holdout.py`` (task arguments, item
draws, statistic names and definitions).
"""

from __future__ import annotations

import math
from typing import Sequence

import numpy as np
import torch
import torch.nn.functional as F

from ..core import EvalCtx, TaskResult, exposure, log_probs, store_record


def _stats(logp: torch.Tensor, tgt: torch.Tensor, which: Sequence[str], top_p: float,
           rep_l: Sequence[int]) -> dict[str, torch.Tensor]:
    """Per-sequence statistics of log-probs (B, T, V) against targets (B, T)."""
    out: dict[str, torch.Tensor] = {}
    if "nll" in which:
        out["nll"] = -logp.gather(-1, tgt.unsqueeze(-1)).squeeze(-1).mean(1)
    if "entropy" in which or "top_p_support" in which:
        p = logp.exp()
        if "entropy" in which:
            out["entropy"] = -(p * logp).sum(-1).mean(1)
        if "top_p_support" in which:
            ps = p.sort(-1, descending=True).values
            before = ps.cumsum(-1) - ps                 # mass strictly before each ranked token
            out["top_p_support"] = (before < top_p).sum(-1).float().mean(1)
    if "rep_at_l" in which:
        pred = logp.argmax(-1)
        for l in rep_l:
            # window of the l text tokens before each position (-1 = before the text)
            prev = F.pad(tgt, (l, 0), value=-1).unfold(1, l, 1)[:, :-1]
            rep = (prev == pred.unsqueeze(-1)).any(-1).float().mean(1)
            gold = (prev == tgt.unsqueeze(-1)).any(-1).float().mean(1)
            out.update({f"rep_{l}": rep, f"gold_rep_{l}": gold, f"rep_excess_{l}": rep - gold})
    return out


def run(ctx: EvalCtx, data_dir: str, shards: list[str] | None = None, n_seq: int = 128,
        context_len: int | list[int] = 2048, batch_size: int = 4,
        metrics: Sequence[str] = ("nll", "entropy", "top_p_support", "rep_at_l"), top_p: float = 0.9,
        rep_l: Sequence[int] = (32, 128)) -> TaskResult:
    unknown = set(metrics) - {"nll", "entropy", "top_p_support", "rep_at_l"}
    if unknown:
        raise ValueError(f"holdout: unknown metrics {sorted(unknown)}")
    store = ctx.store(data_dir, shards)
    lengths = sorted({int(x) for x in (context_len if isinstance(context_len, (list, tuple)) else [context_len])})
    draws = ctx.draws(store, "windows")
    windows = [draws.window(lengths[-1]) for _ in range(n_seq)]
    gen = ctx.subject.generator
    limit = gen.model.max_stream_len
    rep_l = tuple(int(x) for x in rep_l)
    res = TaskResult()
    done, skipped = [], []
    for L in lengths:
        if limit is not None and L > limit:
            skipped.append(L)
            continue
        per: dict[str, list[float]] = {}
        for b0 in range(0, n_seq, batch_size):
            ids = torch.from_numpy(np.stack([draws.read(s, st, L) for s, st in windows[b0:b0 + batch_size]]))
            logp = log_probs(gen, ids)
            for k, v in _stats(logp, ids[:, 1:].to(logp.device), metrics, top_p, rep_l).items():
                per.setdefault(k, []).extend(v.cpu().tolist())
            del logp
        for k, v in per.items():
            res.add_items(f"{k}@{L}", v)
        if "nll" in per:
            res.scalars[f"ppl@{L}"] = math.exp(res.scalars[f"nll@{L}"])
        done.append(L)
        ctx.log(f"  L={L}: " + " ".join(f"{k}={res.scalars[f'{k}@{L}']:.4f}" for k in per))
    res.witness = {"n_seq": n_seq, "lengths": done, "lengths_skipped": skipped, "metrics": list(metrics),
                   "top_p": top_p, "rep_l": list(rep_l),
                   "store": {**store_record(store, tokenizer=True), "total_tokens": store.total_tokens},
                   "exposure": exposure(ctx.subject, store),
                   "windows": [[store.entries[s]["file"], st] for s, st in windows]}
    return res
