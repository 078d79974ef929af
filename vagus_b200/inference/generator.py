"""Stream-state generation over any ``Decodable`` model.

A ``Generator`` owns one token stream per batch row.  Its bookkeeping is a
``_Streams`` record -- rows, capacity, how many tokens the model state has
consumed, and the ``head``: the newest token of every row, which the model
has NOT consumed yet.  A stream is always "model state + head", which gives
the three verbs their meaning:

* ``reset`` opens empty streams (the head is the document-start token when
  the tokenizer has one, so a fresh stream can be continued without a prompt);
* appending tokens (``prefill_ids``) feeds the old head and every new token
  but the last in ONE model call without logits, and the last new token
  becomes the head -- a prompt never materialises vocabulary logits;
* a generation step feeds the head alone, samples from its logits, and the
  sample becomes the head before it is handed out, so a consumer may stop
  at any token with a consistent stream.

Every token is fed exactly once, and logits are computed once per sampled
position.  Generation stops at ``max_new_tokens``, at stream capacity, or
when every row has produced a stop id; the stop test is the only per-token
read of device data, and it is skipped when there are no stop ids, so a
run without stop ids queues all its decode steps without waiting on the GPU.

Batches are (B, L) with equal-length rows (the decode step takes no padding
mask).  ``score_ids`` is teacher-forced scoring through the same decode path
(fresh streams, one feed with logits), so evaluation needs nothing of a model
but the Decodable protocol.

Parity: reference ``infra/inference/generator.py`` (the same verbs and
stream conventions: start token as the fresh head, stop ids, capacity, state
snapshots that resume generation exactly).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Sequence

import torch

from ..models.decodable import Decodable, missing_decodable
from ..utils import infer_device
from .sampling import SamplingConfig, sample


@dataclass
class _Streams:
    rows: int = 0
    capacity: int = 0
    consumed: int = 0                      # tokens held by the model state
    head: torch.Tensor | None = None       # (rows,) int64, not yet consumed

    @property
    def length(self) -> int:
        return self.consumed + (0 if self.head is None else 1)


class Generator:
    """Token streams over a Decodable model, with an optional tokenizer
    (``tokenizers.Tokenizer``) for the text conveniences.  ``start_id`` is
    how a document starts (the head of a fresh stream), ``stop_ids`` how it
    ends (the default of ``SamplingConfig.stop_ids=None``); both belong to
    the tokenizer's stream conventions, not to the model."""

    def __init__(self, model: Decodable, tokenizer=None, start_id: int | None = None,
                 stop_ids: tuple[int, ...] = ()):
        missing = missing_decodable(model)
        if missing:
            raise TypeError(f"{type(model).__name__} does not implement Decodable: missing {missing}")
        self.model = model
        self.tokenizer = tokenizer
        self.start_id = start_id
        self.stop_ids = tuple(int(t) for t in stop_ids)
        self.device = infer_device(model)
        self.rng = torch.Generator(device=self.device)
        self.rng.seed()
        self.streams = _Streams()
        self.stop_reason: str | None = None      # "stop_id" | "max_new_tokens" | "capacity"

    @classmethod
    def from_checkpoint(cls, path, device="cpu", dtype=None, tokenizer_id: str | None = None,
                        with_meta: bool = False):
        """Model, tokenizer and stream conventions from one checkpoint
        (``tokenizer_id`` overrides the checkpoint's record and is required
        when it has none).  ``with_meta`` also returns ``load_model``'s
        record of the checkpoint."""
        from .. import tokenizers
        from ..models.io import load_model
        model, meta = load_model(path, device=device, dtype=dtype)
        tid = tokenizer_id or (meta.get("tokenizer") or {}).get("id")
        if tid is None:
            raise ValueError(f"{path} records no tokenizer; pass tokenizer_id=")
        start_id, stop_ids = tokenizers.stream_conventions(tid)
        gen = cls(model, tokenizers.load(tid), start_id=start_id, stop_ids=stop_ids)
        return (gen, meta) if with_meta else gen

    # ------------------------------------------------------------ bookkeeping --

    @property
    def batch_size(self) -> int:
        return self.streams.rows

    @property
    def max_len(self) -> int:
        return self.streams.capacity

    @property
    def fed_len(self) -> int:
        return self.streams.consumed

    @property
    def pending(self) -> torch.Tensor | None:
        return self.streams.head

    @property
    def stream_len(self) -> int:
        """Tokens per stream, the unconsumed head included."""
        return self.streams.length

    def _capacity(self, requested: int | None) -> int:
        cap = requested if requested is not None else self.model.max_stream_len
        if cap is None:
            raise ValueError("this model has no positional limit: give the stream capacity (max_len)")
        return int(cap)

    def reset(self, batch_size: int = 1, max_len: int | None = None) -> None:
        """Open ``batch_size`` empty streams of capacity ``max_len`` tokens
        (default: the model's ``max_stream_len``)."""
        cap = self._capacity(max_len)
        self.model.reset_cache(batch_size, cap)
        head = None if self.start_id is None else torch.full((batch_size,), self.start_id, dtype=torch.int64,
                                                             device=self.device)
        self.streams = _Streams(rows=batch_size, capacity=cap, consumed=0, head=head)
        self.stop_reason = None

    def export_state(self) -> dict:
        """A snapshot from which ``load_state`` resumes exactly: the model's
        cache, the stream record and the sampling RNG."""
        s = self.streams
        return {"cache": self.model.export_cache(),
                "streams": {"rows": s.rows, "capacity": s.capacity, "consumed": s.consumed,
                            "head": None if s.head is None else s.head.clone()},
                "rng": self.rng.get_state()}

    def load_state(self, state: dict, max_len: int | None = None) -> None:
        rec = state["streams"]
        cap = self._capacity(max_len or rec["capacity"])
        self.model.load_cache(state["cache"], max_cache_len=cap)
        head = rec["head"]
        self.streams = _Streams(rows=rec["rows"], capacity=cap, consumed=rec["consumed"],
                                head=None if head is None else head.to(self.device))
        self.rng.set_state(state["rng"])
        self.stop_reason = None

    # ---------------------------------------------------------------- feeding --

    @torch.no_grad()
    def _consume(self, block: torch.Tensor, logits: bool) -> torch.Tensor | None:
        """Feed ``block`` (rows, L) to the model; (rows, L, V) logits when asked."""
        s = self.streams
        if s.rows == 0:
            raise RuntimeError("no open streams: call reset() first")
        if block.shape[0] != s.rows:
            raise ValueError(f"block has {block.shape[0]} rows, the streams {s.rows}")
        if s.consumed + block.shape[1] > s.capacity:
            raise RuntimeError(f"a stream would hold {s.consumed + block.shape[1]} tokens; its capacity is "
                               f"{s.capacity}")
        if block.shape[1] == 0:
            return None
        out = self.model.decode_step(block, return_logits=logits)
        s.consumed += block.shape[1]
        return out

    def _append(self, ids: torch.Tensor, logits: bool) -> torch.Tensor | None:
        """Append ``ids`` (rows, L >= 1) to the streams: the old head and all
        but the last new token are consumed, the last becomes the head."""
        if ids.dim() != 2 or ids.shape[1] < 1:
            raise ValueError("ids must be (B, L) with L >= 1")
        ids = ids.to(self.device, dtype=torch.int64)
        head = self.streams.head
        block = ids[:, :-1] if head is None else torch.cat([head[:, None], ids[:, :-1]], dim=1)
        out = self._consume(block, logits)
        self.streams.head = ids[:, -1].clone()
        return out

    def prefill_ids(self, ids: torch.Tensor) -> None:
        """Append token ids (B, L) to the streams; no logits are computed."""
        self._append(ids, logits=False)

    def score_ids(self, ids: torch.Tensor) -> torch.Tensor:
        """Teacher-forced logits over fresh streams holding ``ids`` (B, L):
        (B, T, V) where ``[:, t]`` predicts ``ids[:, L - T + t]`` from the
        tokens before it -- T = L with a start token (every token is
        predicted), L - 1 without one.  The streams stay open, as
        ``prefill_ids`` would leave them, so generation may follow."""
        if ids.dim() != 2 or ids.shape[1] < 1:
            raise ValueError("ids must be (B, L) with L >= 1")
        self.reset(ids.shape[0], max_len=ids.shape[1])
        return self._append(ids, logits=True)

    # ------------------------------------------------------------- generation --

    @torch.no_grad()
    def gen_ids_stream(self, cfg: SamplingConfig) -> Iterator[torch.Tensor]:
        """One (B,) int64 tensor per generated position, already part of the
        streams when yielded (stop ids included); the iterator ending is the
        stop, with its cause in ``stop_reason``."""
        s = self.streams
        if s.head is None:
            raise RuntimeError("the streams are empty: prefill a prompt first (this tokenizer has no start token)")
        if cfg.seed is not None:
            self.rng.manual_seed(cfg.seed)
        stops = self.stop_ids if cfg.stop_ids is None else tuple(cfg.stop_ids)
        stop_t = torch.tensor(stops, dtype=torch.int64, device=self.device) if stops else None
        finished = torch.zeros(s.rows, dtype=torch.bool, device=self.device) if stops else None
        self.stop_reason = "max_new_tokens"
        for _ in range(cfg.max_new_tokens):
            if s.consumed >= s.capacity:
                self.stop_reason = "capacity"
                return
            logits = self._consume(s.head[:, None], logits=True)[:, -1]
            tok = sample(logits, cfg, self.rng)
            s.head = tok
            yield tok
            if stop_t is not None:
                finished |= torch.isin(tok, stop_t)
                if bool(finished.all()):             # the one host read per token, only with stop ids
                    self.stop_reason = "stop_id"
                    return

    def gen_ids(self, cfg: SamplingConfig) -> torch.Tensor:
        """(B, N) int64 with N <= ``cfg.max_new_tokens``."""
        toks = list(self.gen_ids_stream(cfg))
        if not toks:
            return torch.empty(self.streams.rows, 0, dtype=torch.int64, device=self.device)
        return torch.stack(toks, dim=1)

    def generate_ids(self, ids: torch.Tensor, cfg: SamplingConfig, max_len: int | None = None) -> torch.Tensor:
        """Fresh streams, ``ids`` as the prompt, the completion out."""
        self.reset(ids.shape[0], max_len)
        self.prefill_ids(ids)
        return self.gen_ids(cfg)

    # ------------------------------------------------------------------- text --

    def _tok(self):
        if self.tokenizer is None:
            raise RuntimeError("this generator has no tokenizer: use the *_ids methods")
        return self.tokenizer

    def encode(self, texts: Sequence[str]) -> torch.Tensor:
        """(B, L) int64 pieces without special tokens (document boundaries
        are the stream's start / stop conventions); rows must have equal
        length."""
        encs = self._tok().encode_batch(list(texts), add_special_tokens=False)
        widths = sorted({len(e.ids) for e in encs})
        if len(widths) != 1:
            raise ValueError(f"prompts must encode to equal lengths (got {widths})")
        return torch.tensor([e.ids for e in encs], dtype=torch.int64, device=self.device)

    def decode(self, ids: torch.Tensor) -> list[str]:
        return self._tok().decode_batch(ids.tolist(), skip_special_tokens=True)

    def prefill(self, texts: Sequence[str] | str) -> None:
        self.prefill_ids(self.encode([texts] if isinstance(texts, str) else texts))

    def gen_stream(self, cfg: SamplingConfig) -> Iterator[list[str]]:
        """Per step, the new text of every row.  A piece alone is not
        always printable (a word marker, half of a multi-byte character), so
        each row's whole continuation is decoded every step and only the part
        that is stable -- no trailing replacement character -- is emitted;
        the rest follows when it completes or at the end."""
        rows = self.streams.rows
        toks: list[list[int]] = [[] for _ in range(rows)]
        shown = [""] * rows

        def delta(final: bool) -> list[str]:
            texts = self.decode(torch.tensor(toks, dtype=torch.int64))
            out = []
            for r, text in enumerate(texts):
                stable = text if final else text.rstrip("�")
                out.append(stable[len(shown[r]):] if stable.startswith(shown[r]) else stable)
                shown[r] = stable
            return out

        for step in self.gen_ids_stream(cfg):
            for r, t in enumerate(step.tolist()):
                toks[r].append(t)
            yield delta(final=False)
        if toks and toks[0]:
            tail = delta(final=True)
            if any(tail):
                yield tail

    def gen(self, cfg: SamplingConfig) -> list[str]:
        return self.decode(self.gen_ids(cfg))

    def generate(self, texts: Sequence[str] | str, cfg: SamplingConfig, max_len: int | None = None) -> list[str]:
        """Fresh streams, text prompts in, text completions out."""
        texts = [texts] if isinstance(texts, str) else list(texts)
        self.reset(len(texts), max_len)
        self.prefill(texts)
        return self.gen(cfg)
