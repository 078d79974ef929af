"""The streaming-inference protocol every registered model implements.

``decode_step(tokens)`` consumes the next block (B, L) of one continuous token
stream whose prefix the state already holds: prefill is the first large block,
L == 1 is single-token decode, L == 0 is a no-op.  ``return_logits=False``
advances the state only (prefill never materialises vocab logits).

Parity: reference ``infra/models/decodable.py:23-46``.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable

import torch

from .cache import WithCache, missing_members


@runtime_checkable
class Decodable(WithCache, Protocol):
    @property
    def max_stream_len(self) -> int | None:
        """Hard bound on the stream length (None: no positional limit)."""
        ...

    def decode_step(self, tokens: torch.Tensor, return_logits: bool = True) -> torch.Tensor | None:
        ...


def missing_decodable(obj) -> list[str]:
    return missing_members(Decodable, obj)
