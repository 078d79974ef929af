"""Repetition in free-running generation, read against real text.

Prompts are document openings (``Draws.document``, salt ``"prompts"``):
``prompt_tokens`` tokens after the document's start token, continued for
``new_tokens`` tokens greedily and with ``seeds`` sampled runs; the
document's own next ``new_tokens`` tokens are the real-text floor at the
same positions.

  rep{n}   seq-rep-n of one continuation: the share of its n-grams that
           repeat an earlier n-gram of it (1 - distinct-n; Welleck et al.,
           2019).  It depends on length and sampling settings, which the
           witness pins; read it against rep{n}_floor.

Items per kind: rep{n}_floor and rep{n}_greedy per prompt, rep{n}_sampled
per (seed, prompt), seed-major.  Samples: every continuation as text.

Parity: reference ``infra/eval/tasks/degeneration.py`` (arguments, draws,
item layout, sampling seeds from ``ctx.torch_seed("sample{s}")``).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from ...inference import SamplingConfig
from ..core import EvalCtx, TaskResult, exposure, store_record


def rep_n(tokens: Sequence[int], n: int) -> float:
    """Share of repeated n-grams among the n-grams of ``tokens``."""
    total = len(tokens) - n + 1
    if total <= 0:
        return 0.0
    distinct = len({tuple(tokens[i:i + n]) for i in range(total)})
    return 1.0 - distinct / total


def run(ctx: EvalCtx, data_dir: str, shards: list[str] | None = None, n_prompts: int = 32,
        prompt_tokens: int = 32, new_tokens: int = 96, seeds: int = 5, sampling: dict | None = None,
        greedy: bool = True, rep_ns: Sequence[int] = (4,), batch_size: int = 32) -> TaskResult:
    sampling = {"temperature": 0.8, "top_p": 0.9, **(sampling or {})}
    store = ctx.store(data_dir, shards)
    draws = ctx.draws(store, "prompts")
    span = 1 + prompt_tokens + new_tokens          # start token + prompt + real continuation
    picks = [draws.document(span) for _ in range(n_prompts)]
    prompts = torch.from_numpy(np.stack([d[1:1 + prompt_tokens] for _, _, d in picks]).astype(np.int64))
    floor = np.stack([d[1 + prompt_tokens:span] for _, _, d in picks]).astype(np.int64)
    gen = ctx.subject.generator
    ns = [int(n) for n in rep_ns]
    res = TaskResult()
    prompt_text = gen.decode(prompts)

    def continue_all(cfg: SamplingConfig) -> np.ndarray:
        parts = [gen.generate_ids(prompts[b:b + batch_size], cfg, max_len=prompt_tokens + new_tokens + 1).cpu()
                 for b in range(0, n_prompts, batch_size)]
        return torch.cat(parts).numpy()

    runs: list[tuple[str, int | None, np.ndarray]] = [("floor", None, floor)]
    if greedy:
        runs.append(("greedy", None, continue_all(SamplingConfig(max_new_tokens=new_tokens, temperature=0,
                                                                stop_ids=()))))
    for s in range(seeds):
        cfg = SamplingConfig(max_new_tokens=new_tokens, stop_ids=(), seed=ctx.torch_seed(f"sample{s}"), **sampling)
        runs.append(("sampled", s, continue_all(cfg)))
    per: dict[str, list[float]] = {}
    for kind, seed, cont in runs:
        texts = gen.decode(torch.from_numpy(cont))
        for p in range(n_prompts):
            row = {"kind": kind, "seed": seed, "prompt_id": p, "prompt": prompt_text[p], "text": texts[p]}
            for n in ns:
                row[f"rep{n}"] = rep_n(cont[p].tolist(), n)
                per.setdefault(f"rep{n}_{kind}", []).append(row[f"rep{n}"])
            res.samples.append(row)
    for k, v in per.items():
        res.add_items(k, v)
    for n in ns:
        f = res.scalars.get(f"rep{n}_floor", 0.0)
        if f"rep{n}_sampled" in res.scalars and f > 0:
            res.scalars[f"rep{n}_sampled_over_floor"] = res.scalars[f"rep{n}_sampled"] / f
    ctx.log("  " + " ".join(f"{k}={v:.4f}" for k, v in res.scalars.items()))
    res.witness = {"n_prompts": n_prompts, "prompt_tokens": prompt_tokens, "new_tokens": new_tokens,
                   "seeds": seeds, "sampling": sampling, "greedy": greedy, "rep_ns": ns,
                   "store": store_record(store), "exposure": exposure(ctx.subject, store),
                   "prompts": [[store.entries[s]["file"], i] for s, i, _ in picks]}
    return res
