"""Sampling configuration and the single logits -> token step (fp32).

top_p keeps a token while the probability mass *before* it is < top_p (the
most likely token always survives); temperature 0 is greedy.

Parity: reference ``infra/inference/sampling.py:8-52``.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import torch


@dataclass(frozen=True)
class SamplingConfig:
    max_new_tokens: int = 128
    temperature: float = 1.0
    top_k: int | None = None
    top_p: float | None = None
    stop_ids: tuple[int, ...] | None = None
    seed: int | None = None

    def __post_init__(self):
        assert self.max_new_tokens >= 0
        assert self.temperature >= 0
        assert self.top_k is None or self.top_k >= 1
        assert self.top_p is None or 0 < self.top_p <= 1

    def asdict(self) -> dict:
        return asdict(self)


def sample(logits: torch.Tensor, cfg: SamplingConfig, rng: torch.Generator | None = None) -> torch.Tensor:
    """logits (B, V) -> token ids (B,) int64."""
    logits = logits.float()
    if cfg.temperature == 0:
        return logits.argmax(dim=-1)
    logits = logits / cfg.temperature
    if cfg.top_k is not None and cfg.top_k < logits.shape[-1]:
        kth = torch.topk(logits, cfg.top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if cfg.top_p is not None and cfg.top_p < 1:
        sl, si = torch.sort(logits, descending=True, dim=-1)
        p = torch.softmax(sl, dim=-1)
        drop = (p.cumsum(-1) - p) >= cfg.top_p
        sl = sl.masked_fill(drop, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(-1, si, sl)
    probs = torch.softmax(logits, dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=rng).squeeze(-1)
