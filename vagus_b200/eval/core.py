"""What an evaluation is made of, shared by the runner and every task.

* ``Subject``: one checkpoint, resolved into a Generator plus its records.
* ``TaskResult``: summary scalars, per-item arrays (paired across subjects
  by position), a witness of what the task did, optional text samples.
* ``EvalCtx``: everything a task may use -- the subject, device / dtype, a
  log, token stores, and randomness derived from (seed, task, salt) alone.
* ``Draws``: the one sampler of evaluation items.  It consumes a numpy
  generator in a fixed pattern (a shard chosen with probability proportional
  to its tokens -- or its documents -- then a uniform position or document
  index in it), so the items of a (seed, task, args) triple are the same for
  every subject and for every framework that follows the same pattern.
* ``log_probs``: the one scorer -- teacher-forced fp32 log-probabilities of
  every token after the first, through the Decodable protocol.

Reproducibility contract (kept identical to the reference so that records
of both frameworks pair item for item): ``rng(salt)`` is
``numpy.random.default_rng`` seeded with the first 8 bytes (little endian)
of SHA-256(``"{seed}/{task}/{salt}"``); ``torch_seed(salt)`` is bytes 8..12
of the same digest modulo 2^31; the draw pattern is ``Draws``'.

Parity: reference ``infra/eval/core.py`` (Subject, TaskResult, EvalCtx,
check_tokenizer, exposure).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable

import numpy as np
import torch

from ..data.loader import TokenStore
from ..inference import Generator


@dataclass
class Subject:
    """A checkpoint under evaluation: ``meta`` is ``load_model``'s record
    (model_name / args, tokenizer, step, tokens_seen, format); ``run_meta``
    the training run's meta.json when one is known (its data record says
    what the model was trained on)."""
    label: str
    path: Path
    sha256: str
    meta: dict
    generator: Generator
    run_meta: dict | None = None

    @property
    def model(self):
        return self.generator.model

    @property
    def param_count(self) -> int:
        return sum(p.numel() for p in self.model.parameters())

    def identity(self) -> dict:
        """The subject's entry in the record's meta.json."""
        ckpt_keys = ("model_name", "model_args", "tokenizer", "step", "tokens_seen", "format")
        return {"label": self.label, "path": str(self.path), "sha256": self.sha256,
                "checkpoint": {k: self.meta.get(k) for k in ckpt_keys}, "param_count": self.param_count,
                "max_stream_len": self.model.max_stream_len,
                "train_data": (self.run_meta or {}).get("data")}


@dataclass
class TaskResult:
    scalars: dict[str, float] = field(default_factory=dict)
    items: dict[str, list[float]] = field(default_factory=dict)
    witness: dict[str, Any] = field(default_factory=dict)
    samples: list[dict] = field(default_factory=list)

    def add_items(self, key: str, values) -> None:
        """Per-item values under ``key`` and their mean as the scalar."""
        vals = [float(v) for v in values]
        self.items[key] = vals
        self.scalars[key] = float(np.mean(vals)) if vals else float("nan")


_OPEN_STORES: dict[tuple, TokenStore] = {}


def open_store(data_dir, shards=None) -> TokenStore:
    """A token store, opened once per process (memory-mapped shards)."""
    key = (str(Path(data_dir).resolve()), tuple(shards or ()))
    if key not in _OPEN_STORES:
        _OPEN_STORES[key] = TokenStore(data_dir, shards=list(shards) if shards else None)
    return _OPEN_STORES[key]


def check_tokenizer(subject: Subject, store: TokenStore) -> None:
    """Refuse a store tokenized differently from the subject's training data
    (when both record a tokenizer hash)."""
    want = (subject.meta.get("tokenizer") or {}).get("sha256")
    have = (store.manifest.get("tokenizer") or {}).get("sha256")
    if want and have and want != have:
        raise ValueError(f"{subject.label}: trained with tokenizer {want[:8]}, store {store.dir} uses {have[:8]}")


def exposure(subject: Subject, store: TokenStore) -> dict:
    """How often, on average, the subject saw each token of ``store`` during
    training if its windows were uniform over it (tokens seen / store
    tokens), and whether the store is the training run's (source and
    tokenizer hash), when the run's record is known."""
    seen = subject.meta.get("tokens_seen")
    train = (subject.run_meta or {}).get("data")
    same = None
    if train:
        same = (train.get("source") == store.manifest.get("source")
                and (train.get("tokenizer") or {}).get("sha256") == store.manifest["tokenizer"].get("sha256"))
    return {"tokens_seen": seen, "store_tokens": store.total_tokens,
            "expected_views": seen / store.total_tokens if seen else None, "same_store": same,
            "train_total_tokens": train.get("total_tokens") if train else None}


def store_record(store: TokenStore, tokenizer: bool = False) -> dict:
    """A store's identity for a witness."""
    rec = {"dir": str(store.dir.resolve()), "source": store.manifest.get("source")}
    if tokenizer:
        rec["tokenizer"] = store.manifest.get("tokenizer", {}).get("id")
    rec["shards"] = [e["file"] for e in store.entries]
    return rec


class Draws:
    """Evaluation items drawn from a store with one numpy generator.

    Each draw first picks a shard -- proportionally to its tokens
    (``window``) or to its documents (``document``) -- with
    ``rng.choice(n_shards, p=...)``, then a position with
    ``rng.integers(0, hi)``.  Tasks that interleave other draws (key / value
    pairs, slots) use ``rng`` directly between these calls."""

    def __init__(self, store: TokenStore | None, rng: np.random.Generator):
        self.store = store
        self.rng = rng
        self._tok_p = self._docs = self._doc_p = None
        if store is not None:
            w = np.asarray(store.shard_tokens, dtype=np.float64)
            self._tok_p = w / w.sum()

    def window(self, length: int, slack: int = 0) -> tuple[int, int]:
        """(shard, start) of a window of ``length`` tokens; the start is
        uniform in [0, shard tokens - length - slack)."""
        s = int(self.rng.choice(len(self._tok_p), p=self._tok_p))
        return s, int(self.rng.integers(0, self.store.shard_tokens[s] - length - slack))

    def read(self, shard: int, start: int, length: int) -> np.ndarray:
        return self.store.read_window(shard, start, length).astype(np.int64)

    def document(self, min_len: int) -> tuple[int, int, np.ndarray]:
        """(shard, index, tokens) of a document of at least ``min_len``
        tokens; shorter draws are discarded and drawn again."""
        if self._docs is None:
            self._docs = [len(self.store.doc_offsets(s)) - 1 for s in range(len(self.store.entries))]
            w = np.asarray(self._docs, dtype=np.float64)
            self._doc_p = w / w.sum()
        while True:
            s = int(self.rng.choice(len(self._doc_p), p=self._doc_p))
            i = int(self.rng.integers(0, self._docs[s]))
            doc = self.store.doc(s, i)
            if len(doc) >= min_len:
                return s, i, doc


def log_probs(gen: Generator, ids: torch.Tensor) -> torch.Tensor:
    """fp32 log-probabilities (B, L - 1, V) of ``ids[:, 1:]`` given the
    stream before each token (the start token, when the tokenizer has one,
    stands before ``ids[:, 0]``; its prediction of ``ids[:, 0]`` is left
    out, so every subject is scored on the same L - 1 positions)."""
    logits = gen.score_ids(ids)
    if gen.start_id is not None:
        logits = logits[:, 1:]
    return logits.float().log_softmax(-1)


class EvalCtx:
    """What the runner hands a task."""

    def __init__(self, subject: Subject, task: str, seed: int, device: torch.device, dtype: torch.dtype,
                 log: Callable[[str], None]):
        self.subject = subject
        self.task = task
        self.seed = seed
        self.device = device
        self.dtype = dtype
        self.log = log

    def _digest(self, salt: str) -> bytes:
        return hashlib.sha256(f"{self.seed}/{self.task}/{salt}".encode()).digest()

    def rng(self, salt: str = "") -> np.random.Generator:
        """A numpy generator determined by (seed, task, salt) only."""
        return np.random.default_rng(int.from_bytes(self._digest(salt)[:8], "little"))

    def torch_seed(self, salt: str = "") -> int:
        """A sampling seed determined by (seed, task, salt) only."""
        return int.from_bytes(self._digest(salt)[8:12], "little") % (2 ** 31)

    def store(self, data_dir, shards=None) -> TokenStore:
        st = open_store(data_dir, shards)
        check_tokenizer(self.subject, st)
        return st

    def draws(self, store: TokenStore | None, salt: str) -> Draws:
        return Draws(store, self.rng(salt))
