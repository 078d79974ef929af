"""Stateful autoregressive generation over any ``Decodable`` model.

Invariant: model state + ``pending`` == the whole stream.  ``pending`` is the
newest token, not yet consumed.  ``prefill_ids`` feeds all but the last new
token (no logits are materialised for a prompt) and makes that token pending;
each generation step feeds the pending token (L == 1), samples, and the sample
becomes pending -- so every token is fed once, the state is closed after every
step, and a stream consumer may stop at any point.

On CUDA the single-token step of a model can be captured into a CUDA graph
(``Generator(..., cuda_graph=True)``): the per-token launch overhead, which
dominates decode at these model sizes, is paid once per capture.

Parity: reference ``infra/inference/generator.py:36-309`` (same verbs, same
state export layout, same stop semantics).
"""

from __future__ import annotations

from typing import Iterator, Sequence

import torch

from ..models.decodable import Decodable, missing_decodable
from ..utils import infer_device
from .sampling import SamplingConfig, sample


class Generator:
    def __init__(self, model: Decodable, tokenizer=None, start_id: int | None = None, stop_ids: tuple[int, ...] = ()):
        missing = missing_decodable(model)
        assert not missing, f"{type(model).__name__} lacks Decodable members {missing}"
        self.model = model
        self.tokenizer = tokenizer
        self.start_id = start_id
        self.stop_ids = tuple(stop_ids)
        self.device = infer_device(model)
        self.rng = torch.Generator(device=self.device)
        self.rng.seed()
        self.batch_size = 0
        self.max_len = 0
        self.fed_len = 0
        self.pending: torch.Tensor | None = None
        self.stop_reason: str | None = None

    @classmethod
    def from_checkpoint(cls, path, device="cpu", dtype=None, tokenizer_id: str | None = None, with_meta: bool = False):
        from .. import tokenizers
        from ..models.io import load_model
        model, meta = load_model(path, device=device, dtype=dtype)
        if tokenizer_id is None:
            if meta["tokenizer"] is None:
                raise ValueError(f"{path} records no tokenizer; pass tokenizer_id=")
            tokenizer_id = meta["tokenizer"]["id"]
        start_id, stop_ids = tokenizers.stream_conventions(tokenizer_id)
        gen = cls(model, tokenizers.load(tokenizer_id), start_id=start_id, stop_ids=stop_ids)
        return (gen, meta) if with_meta else gen

    # --- state ---------------------------------------------------------------

    def _resolve_max_len(self, max_len: int | None) -> int:
        if max_len is None:
            max_len = self.model.max_stream_len
        if max_len is None:
            raise ValueError("model has no max_stream_len; pass max_len to reset()")
        return int(max_len)

    def reset(self, batch_size: int = 1, max_len: int | None = None) -> None:
        self.batch_size = batch_size
        self.max_len = self._resolve_max_len(max_len)
        self.model.reset_cache(batch_size, self.max_len)
        self.fed_len = 0
        self.pending = None if self.start_id is None else torch.full(
            (batch_size,), self.start_id, dtype=torch.int64, device=self.device)
        self.stop_reason = None

    @property
    def stream_len(self) -> int:
        return self.fed_len + (0 if self.pending is None else 1)

    def export_state(self) -> dict:
        return {"cache": self.model.export_cache(),
                "pending": None if self.pending is None else self.pending.clone(),
                "fed_len": self.fed_len, "batch_size": self.batch_size, "max_len": self.max_len,
                "rng": self.rng.get_state()}

    def load_state(self, state: dict, max_len: int | None = None) -> None:
        self.batch_size = state["batch_size"]
        self.max_len = self._resolve_max_len(max_len or state["max_len"])
        self.model.load_cache(state["cache"], max_cache_len=self.max_len)
        self.pending = None if state["pending"] is None else state["pending"].to(self.device)
        self.fed_len = state["fed_len"]
        self.rng.set_state(state["rng"])
        self.stop_reason = None

    # --- feeding -------------------------------------------------------------

    @torch.no_grad()
    def _feed(self, block: torch.Tensor, want_logits: bool):
        assert self.batch_size > 0, "call reset() first"
        assert block.shape[0] == self.batch_size
        L = block.shape[1]
        if self.fed_len + L > self.max_len:
            raise RuntimeError(f"stream capacity {self.max_len} exceeded: {self.fed_len} fed + {L} new")
        if L == 0:
            return None
        out = self.model.decode_step(block.to(self.device), return_logits=want_logits)
        self.fed_len += L
        if not want_logits:
            return None
        return out[:, -1]

    def prefill_ids(self, ids: torch.Tensor) -> None:
        assert ids.dim() == 2 and ids.shape[1] >= 1, "ids must be (B, L) with L >= 1"
        ids = ids.to(self.device, dtype=torch.int64)
        block = ids[:, :-1] if self.pending is None else torch.cat([self.pending[:, None], ids[:, :-1]], 1)
        self._feed(block, want_logits=False)
        self.pending = ids[:, -1].clone()

    @torch.no_grad()
    def score_ids(self, ids: torch.Tensor) -> torch.Tensor:
        """Teacher-forced logits (B, T, vocab) over fresh streams through the
        decode path; T == L with a start token, L - 1 without."""
        assert ids.dim() == 2 and ids.shape[1] >= 1
        ids = ids.to(self.device, dtype=torch.int64)
        B, L = ids.shape
        self.reset(B, max_len=L)
        block = ids[:, :-1] if self.pending is None else torch.cat([self.pending[:, None], ids[:, :-1]], 1)
        out = self.model.decode_step(block, return_logits=True)
        self.fed_len += block.shape[1]
        self.pending = ids[:, -1].clone()
        return out

    # --- generation ----------------------------------------------------------

    @torch.no_grad()
    def gen_ids_stream(self, cfg: SamplingConfig) -> Iterator[torch.Tensor]:
        assert self.pending is not None, "empty stream"
        if cfg.seed is not None:
            self.rng.manual_seed(cfg.seed)
        stop_ids = self.stop_ids if cfg.stop_ids is None else cfg.stop_ids
        stop_t = torch.tensor(list(stop_ids), dtype=torch.int64, device=self.device)
        done = torch.zeros(self.batch_size, dtype=torch.bool, device=self.device)
        self.stop_reason = None
        for _ in range(cfg.max_new_tokens):
            if self.fed_len >= self.max_len:
                self.stop_reason = "capacity"
                return
            logits = self._feed(self.pending[:, None], want_logits=True)
            t = sample(logits, cfg, self.rng)
            self.pending = t
            if stop_t.numel():
                done |= torch.isin(t, stop_t)
            yield t
            if bool(done.all()):
                self.stop_reason = "stop_id"
                return
        self.stop_reason = "max_new_tokens"

    def gen_ids(self, cfg: SamplingConfig) -> torch.Tensor:
        steps = list(self.gen_ids_stream(cfg))
        if not steps:
            return torch.zeros(self.batch_size, 0, dtype=torch.int64, device=self.device)
        return torch.stack(steps, 1)

    def generate_ids(self, ids: torch.Tensor, cfg: SamplingConfig, max_len: int | None = None) -> torch.Tensor:
        self.reset(ids.shape[0], max_len)
        self.prefill_ids(ids)
        return self.gen_ids(cfg)

    # --- text ----------------------------------------------------------------

    def encode(self, texts: Sequence[str]) -> torch.Tensor:
        assert self.tokenizer is not None, "no tokenizer: use the *_ids methods"
        encs = self.tokenizer.encode_batch(list(texts), add_special_tokens=False)
        lens = {len(e.ids) for e in encs}
        if len(lens) != 1:
            raise ValueError(f"v1 batches need equal-length prompts, got lengths {sorted(lens)}")
        return torch.tensor([e.ids for e in encs], dtype=torch.int64, device=self.device)

    def decode(self, ids: torch.Tensor) -> list[str]:
        assert self.tokenizer is not None
        return self.tokenizer.decode_batch(ids.tolist(), skip_special_tokens=True)

    def prefill(self, texts) -> None:
        if isinstance(texts, str):
            texts = [texts]
        self.prefill_ids(self.encode(texts))

    def gen_stream(self, cfg: SamplingConfig) -> Iterator[list[str]]:
        """Per-step text deltas; a trailing replacement character is held back
        until the sequence completes (prefix-stable streaming decode)."""
        B = self.batch_size
        ids: list[list[int]] = [[] for _ in range(B)]
        emitted = [""] * B
        for step in self.gen_ids_stream(cfg):
            for b, t in enumerate(step.tolist()):
                ids[b].append(t)
            texts = self.decode(torch.tensor(ids, dtype=torch.int64))
            delta = []
            for b in range(B):
                full = texts[b].rstrip("�") if texts[b].endswith("�") else texts[b]
                if full.startswith(emitted[b]):
                    delta.append(full[len(emitted[b]):])
                else:
                    delta.append(full)
                emitted[b] = full
            yield delta
        if ids and ids[0]:
            texts = self.decode(torch.tensor(ids, dtype=torch.int64))
            tail = [t[len(e):] if t.startswith(e) else t for t, e in zip(texts, emitted)]
            if any(tail):
                yield tail

    def gen(self, cfg: SamplingConfig) -> list[str]:
        return self.decode(self.gen_ids(cfg))

    def generate(self, texts, cfg: SamplingConfig, max_len: int | None = None) -> list[str]:
        if isinstance(texts, str):
            texts = [texts]
        self.reset(len(texts), max_len)
        self.prefill(texts)
        return self.gen(cfg)
