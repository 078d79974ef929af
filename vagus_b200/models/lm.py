"""Shared skeleton of every registered language model:

    embedding -> blocks -> rms_head -> head (tied to the embedding by default)

plus the Decodable verbs, which just walk the blocks.  The concrete models
(``TransformerPP``, ``GDNLM``) choose the mixer of each block, the optimizer
split and the FLOP model.

Parity: the forward / decode / cache methods shared by reference
``infra/models/transformer_pp.py:86-139`` and ``infra/models/gdn_lm.py:180-262``.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import ops
from .decodable import Decodable
from .norm import RMSNorm


class CausalLM(nn.Module, Decodable):
    embedding: nn.Embedding
    blocks: nn.ModuleList
    rms_head: RMSNorm
    head: nn.Linear
    config: dict

    def _finish(self, vocab_size: int, dim: int, rmsnorm_eps: float, tie_embedding: bool) -> None:
        self.rms_head = RMSNorm(dim, rmsnorm_eps)
        self.head = nn.Linear(dim, vocab_size, bias=False)
        nn.init.normal_(self.embedding.weight, std=0.02)
        if tie_embedding:
            self.head.weight = self.embedding.weight
        else:
            nn.init.normal_(self.head.weight, std=0.02)

    @classmethod
    def from_config(cls, config: dict):
        return cls(**config)

    def compile_blocks(self):
        """Kept for recipe compatibility (``compile: true``).  The sm_100a path
        fuses by hand, so nothing is handed to a tracing compiler."""
        return self

    def hidden(self, tokens: torch.Tensor, is_causal: bool = True) -> torch.Tensor:
        x = ops.embedding(tokens, self.embedding.weight)
        for blk in self.blocks:
            x = blk(x, is_causal)
        return self.rms_head(x, out_dtype=torch.bfloat16 if ops.kernels_active(x) else None)

    def forward(self, tokens, is_causal: bool = True, return_hidden: bool = False):
        h = self.hidden(tokens, is_causal)
        if return_hidden:
            return h
        return ops.linear(h, self.head.weight)

    # --- streaming ---------------------------------------------------------

    def reset_cache(self, batch_size: int, max_cache_len: int):
        for blk in self.blocks:
            blk.reset_cache(batch_size, max_cache_len)

    def load_cache(self, cache: dict, max_cache_len: int):
        for blk, c in zip(self.blocks, cache["blocks"], strict=True):
            blk.load_cache(c, max_cache_len=max_cache_len)

    def export_cache(self) -> dict:
        return {"blocks": [blk.export_cache() for blk in self.blocks]}

    @torch.no_grad()
    def decode_step(self, tokens, return_logits: bool = True):
        x = self.embedding(tokens)
        for blk in self.blocks:
            x = blk.decode_step(x)
        if not return_logits:
            return None
        return ops.linear(self.rms_head(x), self.head.weight)
