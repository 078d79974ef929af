"""Transformer++: pre-norm softmax-attention blocks with RoPE and SwiGLU.

Parity: reference ``infra/models/transformer_pp.py:14-183``.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import nn

from .attention import SoftmaxAttention
from .block import Block
from .lm import CausalLM
from .rope import RoPE


class TransformerPP(CausalLM):
    def __init__(self, vocab_size: int, dim: int, head_dim: int, context_len: int, layer_count: int,
                 ffn_hidden_dim: int | None = None, kv_head_count: int | None = None,
                 rmsnorm_eps: float = 1e-6, rope_base: float = 10000, tie_embedding: bool = True,
                 qk_norm: bool = False):
        super().__init__()
        self.config: dict[str, Any] = dict(
            vocab_size=vocab_size, dim=dim, head_dim=head_dim, context_len=context_len,
            layer_count=layer_count, ffn_hidden_dim=ffn_hidden_dim, kv_head_count=kv_head_count,
            rmsnorm_eps=rmsnorm_eps, rope_base=rope_base, tie_embedding=tie_embedding, qk_norm=qk_norm)
        assert dim % head_dim == 0
        self.embedding = nn.Embedding(vocab_size, dim)
        self.rope = RoPE(dim, head_dim, context_len, base=rope_base)
        heads = dim // head_dim
        self.blocks = nn.ModuleList([
            Block(dim=dim, ffn_hidden_dim=ffn_hidden_dim, rmsnorm_eps=rmsnorm_eps, layer_count=layer_count,
                  mixer=SoftmaxAttention(dim=dim, head_count=heads, kv_head_count=kv_head_count, v_dim_mult=1,
                                         short_conv_size=None, qk_norm=qk_norm, rope=self.rope, init_std=0.02,
                                         layer_count=layer_count))
            for _ in range(layer_count)])
        self._finish(vocab_size, dim, rmsnorm_eps, tie_embedding)

    @property
    def max_stream_len(self) -> int:
        return int(self.config["context_len"])

    def param_groups(self) -> dict[str, list[nn.Parameter]]:
        """Muon on the block matrices; AdamW (decayed) on other matrices; no
        decay on vectors."""
        muon = [p for p in self.blocks.parameters() if p.requires_grad and p.dim() == 2]
        ids = {id(p) for p in muon}
        decay = [p for p in self.parameters() if p.requires_grad and id(p) not in ids and p.dim() >= 2]
        no_decay = [p for p in self.parameters() if p.requires_grad and p.dim() < 2]
        return {"muon": muon, "adamw_decay": decay, "adamw_no_decay": no_decay}

    def attn_flops_per_token(self, context_len: int) -> float:
        """PaLM 12 * layers * d * L attention matmul FLOPs (fwd + bwd)."""
        return float(12 * int(self.config["layer_count"]) * int(self.config["dim"]) * context_len)

    def metric_hooks(self) -> dict:
        return {"slow": [self._metric_max_attn_logit]}

    @torch.no_grad()
    def _metric_max_attn_logit(self, ctx) -> dict:
        tokens = ctx.last_batch
        if tokens is None:
            return {}
        x = self.embedding(tokens[:1])
        worst = None
        for blk in self.blocks:
            h = blk.rmsnorm1(x)
            m = blk.att.max_attn_logit(h)
            worst = m if worst is None else torch.maximum(worst, m)
            x = x + blk.att(h)
            x = x + blk.ffn(blk.rmsnorm2(x))
        return {} if worst is None else {"attn_logit_max": float(worst)}
