"""The token-mixer protocol: what a Block needs from the module it wraps.

A mixer maps (B, L, dim) -> (B, L, dim), statelessly in ``forward`` and against
its own state in ``decode_step``.  ``decode_step(x)`` consumes the next block
of a stream whose prefix the state already holds: L == 1 is single-token
decode, a large first block is prefill, L == 0 is a no-op.

Parity: reference ``infra/components/mixer.py:21-42``.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable

import torch

from .cache import WithCache, missing_members


@runtime_checkable
class Mixer(WithCache, Protocol):
    def forward(self, x: torch.Tensor, is_causal: bool = True) -> torch.Tensor:
        """Stateless training / full-sequence path."""
        ...

    def __call__(self, x: torch.Tensor, is_causal: bool = True) -> torch.Tensor:
        """``forward`` through nn.Module's hook machinery (what a Block calls)."""
        ...

    def decode_step(self, x: torch.Tensor) -> torch.Tensor:
        """Consume the next (B, L, dim) block of the stream, advancing the state."""
        ...


def missing_mixer(obj) -> list[str]:
    return missing_members(Mixer, obj)
