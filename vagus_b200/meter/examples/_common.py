"""Shared plumbing of the probes: checkpoints, token windows, and a walk over
a model's blocks that hands each block's mixer input to a visitor."""

from __future__ import annotations

import torch


def parse_ckpts(items: list[str]) -> dict[str, str]:
    """NAME=path pairs (a bare path is named by its position)."""
    out = {}
    for i, it in enumerate(items):
        name, _, path = it.partition("=")
        out[name if path else f"m{i}"] = path or name
    return out


def windows(data_dir: str, context_len: int, batch: int, batches: int, seed: int = 0):
    """``batches`` (batch, context_len) token tensors from a token store."""
    from ...data.loader import TokenStore, WindowLoader
    loader = WindowLoader(TokenStore(data_dir), context_len, batch, seed=seed, prefetch=0)
    it = iter(loader)
    return [next(it)[0] for _ in range(batches)]


def mixers(att):
    """(softmax attention or None, linear attention or None) of a block's mixer."""
    from ...models.attention import SoftmaxAttention
    from ...models.gdn import GatedDeltaNet
    from ...models.parallel_mixer import ParallelMixer
    if isinstance(att, ParallelMixer):
        return att.att, att.la
    if isinstance(att, SoftmaxAttention):
        return att, None
    if isinstance(att, GatedDeltaNet):
        return None, att
    return None, None


@torch.no_grad()
def walk(model, tokens, visit) -> None:
    """visit(layer, block, h) with h = the block's normalised mixer input."""
    x = model.embedding(tokens)
    for i, blk in enumerate(model.blocks):
        visit(i, blk, blk.rmsnorm1(x))
        x = blk(x)
