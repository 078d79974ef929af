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


def decode_bench(layer, x, prefill: int, steps: int, *, iters: int = 5) -> dict:
    """Streaming timings of one mixer layer on input x (B, prefill + steps, D):
    the prefill of ``prefill`` tokens through the cache, and the per-token
    latency of ``steps`` single-token decode steps after it (each timed run
    restores the post-prefill cache first; that copy is included)."""
    from ..core import bench
    B = x.shape[0]
    cap = prefill + steps

    @torch.no_grad()
    def pre():
        layer.reset_cache(B, cap)
        return layer.decode_step(x[:, :prefill])

    pre()
    snap = layer.export_cache()

    @torch.no_grad()
    def dec():
        layer.load_cache(snap, cap)
        out = None
        for t in range(prefill, cap):
            out = layer.decode_step(x[:, t:t + 1])
        return out

    rp = bench(pre, name="prefill", device=x.device, warmup=1, iters=iters)
    rd = bench(dec, name="decode", device=x.device, warmup=1, iters=iters)
    if rp.failed or rd.failed:
        raise RuntimeError(rp.error or rd.error)
    per_tok = rd.mean_ms / max(1, steps)
    return {"prefill_ms": rp.mean_ms, "prefill_tok_s": B * prefill / (rp.mean_ms * 1e-3),
            "decode_ms_per_token": per_tok, "decode_tok_s": B / (per_tok * 1e-3)}


def render_decode(name: str, r: dict) -> str:
    return (f"  {name:<12} prefill {r['prefill_ms']:8.3f} ms ({r['prefill_tok_s'] / 1e3:8.1f}K tok/s)   "
            f"decode {r['decode_ms_per_token'] * 1e3:8.1f} us/token ({r['decode_tok_s'] / 1e3:7.1f}K tok/s)")
