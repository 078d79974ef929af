"""The nouns of an evaluation run, shared by the runner and the tasks.

Subject   one checkpoint resolved into (generator, meta, sha256)
TaskResult scalars, per-item arrays (paired across subjects), witness, samples
EvalCtx   what a task may touch: RNGs derived from (seed, task, salt) only --
          never from the subject -- so every subject sees the same items

Parity: reference ``infra/eval/core.py:15-142``.
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
        return {"label": self.label, "path": str(self.path), "sha256": self.sha256,
                "checkpoint": {k: self.meta.get(k) for k in
                               ("model_name", "model_args", "tokenizer", "step", "tokens_seen", "format")},
                "param_count": self.param_count, "max_stream_len": self.model.max_stream_len,
                "train_data": (self.run_meta or {}).get("data")}


@dataclass
class TaskResult:
    scalars: dict[str, float] = field(default_factory=dict)
    items: dict[str, list[float]] = field(default_factory=dict)
    witness: dict[str, Any] = field(default_factory=dict)
    samples: list[dict] = field(default_factory=list)


_STORES: dict[tuple, TokenStore] = {}


def open_store(data_dir, shards=None) -> TokenStore:
    key = (str(Path(data_dir).resolve()), tuple(shards) if shards else None)
    if key not in _STORES:
        _STORES[key] = TokenStore(data_dir, shards=list(shards) if shards else None)
    return _STORES[key]


class EvalCtx:
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
        return np.random.default_rng(int.from_bytes(self._digest(salt)[:8], "little"))

    def torch_seed(self, salt: str = "") -> int:
        return int.from_bytes(self._digest(salt)[8:12], "little") % (2 ** 31)

    def store(self, data_dir, shards=None) -> TokenStore:
        store = open_store(data_dir, shards)
        check_tokenizer(self.subject, store)
        return store


def check_tokenizer(subject: Subject, store: TokenStore) -> None:
    mine = (subject.meta.get("tokenizer") or {}).get("sha256")
    theirs = store.manifest.get("tokenizer", {}).get("sha256")
    if mine and theirs and mine != theirs:
        raise ValueError(f"{subject.label}: checkpoint tokenizer {mine[:8]} != store tokenizer {theirs[:8]} "
                         f"({store.dir})")


def exposure(subject: Subject, store: TokenStore) -> dict:
    seen = subject.meta.get("tokens_seen")
    train = (subject.run_meta or {}).get("data")
    same = None
    if train:
        same = (train.get("source") == store.manifest.get("source")
                and (train.get("tokenizer") or {}).get("sha256") == store.manifest["tokenizer"].get("sha256"))
    return {"tokens_seen": seen, "store_tokens": store.total_tokens,
            "expected_views": (seen / store.total_tokens) if seen else None, "same_store": same,
            "train_total_tokens": train.get("total_tokens") if train else None}


def sha256_file(path, chunk: int = 1 << 23) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while b := f.read(chunk):
            h.update(b)
    return h.hexdigest()
