"""Associative recall in the MQAR style (Arora et al., Zoology): k key/value
pairs planted in a context of L tokens, every key asked again at the end,
the value scored teacher-forced.  Deterministic (no sampling); a (length,
pairs) cell beyond the subject's ``max_stream_len`` is skipped and listed.

One sequence, as token ids:

  body  (L - 4k tokens): noise with k lines ``key : value \\n`` written over
        it at random positions that are multiples of 4;
  tail  (4k tokens): ``key : value \\n`` for every pair, in random order.

At the value position of every tail line: acc (the argmax is the value),
logprob (log p(value)), copy (the argmax is one of this sequence's values --
the model copies, right or wrong; 1/k is chance given copying).  Keys and
values are distinct word-like tokens (a word-start marker followed by
lower-case letters); noise is real text from the store (``noise: text``)
or uniform draws from the word pool (``random``).  Zero-shot on a
pretrained LM this measures in-context copying; compare subjects that share
a tokenizer.

Draw pattern per sequence (salt ``"sequences"``, cells in argument order,
drawn even for skipped cells so later cells see the same stream):
``rng.choice(pool, 2k, replace=False)`` (keys then values), the noise window
(``Draws.window``) or ``rng.choice(pool, body)``, the slots
``sort(rng.choice(body // 4, k, replace=False)) * 4``, the tail order
``rng.permutation(k)``.

Parity: reference ``infra/eval/tasks/recall_probe.py`` (arguments, sequence
layout, draw pattern, item names).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from ..core import EvalCtx, TaskResult, exposure, store_record


def word_pool(tokenizer, vocab_size: int, min_len: int = 5) -> list[int]:
    """Ids of word-start pieces longer than ``min_len`` characters made of
    lower-case letters, below ``vocab_size``, sorted."""
    out = []
    for piece, i in tokenizer.get_vocab().items():
        word = piece[1:]
        if i < vocab_size and piece[:1] == "▁" and len(piece) > min_len and word.isalpha() and word.islower():
            out.append(i)
    return sorted(out)


def _line(key: int, value: int, colon: int, nl: int) -> tuple[int, int, int, int]:
    return key, colon, value, nl


def run(ctx: EvalCtx, lengths: Sequence[int] = (256, 1024, 4096), kv_pairs: Sequence[int] = (8, 32),
        n: int = 64, noise: str = "text", data_dir: str | None = None, shards: list[str] | None = None,
        batch_size: int = 4, pool: list[int] | None = None, seps: list[int] | None = None) -> TaskResult:
    if noise not in ("text", "random"):
        raise ValueError(f"recall_probe: noise must be 'text' or 'random', not {noise!r}")
    gen = ctx.subject.generator
    vocab_size = int(ctx.subject.meta["model_args"]["vocab_size"])
    ids_pool = word_pool(gen.tokenizer, vocab_size) if pool is None else list(range(int(pool[0]), int(pool[1])))
    if seps is None:
        vocab = gen.tokenizer.get_vocab()
        if ":" not in vocab or "<0x0A>" not in vocab:
            raise ValueError("recall_probe: the tokenizer has no ':' / newline pieces; pass seps=[colon, newline]")
        colon, nl = vocab[":"], vocab["<0x0A>"]
    else:
        colon, nl = int(seps[0]), int(seps[1])
    store = ctx.store(data_dir, shards) if noise == "text" else None
    draws = ctx.draws(store, "sequences")
    rng = draws.rng
    limit = gen.model.max_stream_len
    # position of a tail value in the scored logits: score_ids predicts every
    # token with a start token, all but the first without one
    shift = 0 if gen.start_id is not None else 1
    res = TaskResult()
    cells, skipped = [], []
    for L in (int(x) for x in lengths):
        for k in (int(x) for x in kv_pairs):
            body = L - 4 * k
            if body < 4 * k:
                raise ValueError(f"recall_probe: L={L} cannot hold {k} pairs")
            cell = f"L{L}_p{k}"
            seqs, asked, vals = [], [], []
            for _ in range(n):
                kv = rng.choice(ids_pool, 2 * k, replace=False)
                keys, values = kv[:k], kv[k:]
                base = draws.read(*draws.window(body), body) if store is not None \
                    else rng.choice(ids_pool, body).astype(np.int64)
                for j, pos in enumerate(np.sort(rng.choice(body // 4, k, replace=False)) * 4):
                    base[pos:pos + 4] = _line(keys[j], values[j], colon, nl)
                order = rng.permutation(k)
                tail = np.array([t for j in order for t in _line(keys[j], values[j], colon, nl)], dtype=np.int64)
                seqs.append(np.concatenate([base, tail]))
                asked.append(values[order])
                vals.append(values)
            if limit is not None and L > limit:
                skipped.append(cell)
                continue
            at = torch.tensor([body + 4 * q + 2 - shift for q in range(k)])
            acc, lp, copy = [], [], []
            for b0 in range(0, n, batch_size):
                logits = gen.score_ids(torch.from_numpy(np.stack(seqs[b0:b0 + batch_size])))
                sel = logits[:, at.to(logits.device)].float().log_softmax(-1)        # (B, k, V)
                del logits
                want = torch.from_numpy(np.stack(asked[b0:b0 + batch_size])).to(sel.device)
                have = torch.from_numpy(np.stack(vals[b0:b0 + batch_size])).to(sel.device)
                top = sel.argmax(-1)
                acc += (top == want).float().mean(1).tolist()
                lp += sel.gather(-1, want.unsqueeze(-1)).squeeze(-1).mean(1).tolist()
                copy += (top.unsqueeze(-1) == have.unsqueeze(1)).any(-1).float().mean(1).tolist()
            for name, v in (("acc", acc), ("logprob", lp), ("copy", copy)):
                res.add_items(f"{name}_{cell}", v)
            cells.append(cell)
            ctx.log(f"  {cell}: acc={np.mean(acc):.3f} copy={np.mean(copy):.3f} logprob={np.mean(lp):.3f}")
    if cells:
        res.scalars["acc"] = float(np.mean([res.scalars[f"acc_{c}"] for c in cells]))
    res.witness = {"lengths": list(lengths), "kv_pairs": list(kv_pairs), "n": n, "noise": noise, "cells": cells,
                   "cells_skipped": skipped, "pool_size": len(ids_pool), "seps": [colon, nl],
                   "chance": {f"p{int(k)}": 1.0 / int(k) for k in kv_pairs},
                   "store": None if store is None else store_record(store),
                   "exposure": None if store is None else exposure(ctx.subject, store)}
    return res
