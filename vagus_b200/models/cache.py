"""The streaming-state interface shared by mixers, blocks and models.

A mixer's KV cache or recurrent matrix, a block (which forwards to its mixer)
and a model (which forwards to its blocks) all expose the same three verbs.

Parity: reference ``infra/components/cache.py:11-37``.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable


@runtime_checkable
class WithCache(Protocol):
    def reset_cache(self, batch_size: int, max_cache_len: int) -> None:
        """Allocate an empty state for ``batch_size`` streams.  A growing state
        (KV cache) holds at most ``max_cache_len`` tokens; a fixed-size state
        accepts and ignores the bound."""
        ...

    def export_cache(self) -> dict:
        """A compact, self-contained copy of the state (tensors cloned)."""
        ...

    def load_cache(self, cache: dict, max_cache_len: int) -> None:
        """Restore an exported state, allocating room for ``max_cache_len``."""
        ...


def missing_members(protocol, obj) -> list[str]:
    """Members of ``protocol`` that ``obj`` lacks (empty list = conforms).

    ``isinstance`` against a runtime-checkable Protocol does a static attribute
    lookup that misses what ``nn.Module.__getattr__`` resolves (submodules,
    buffers), so the duck-typed check walks the protocol's attribute set."""
    return [name for name in sorted(protocol.__protocol_attrs__) if not hasattr(obj, name)]
