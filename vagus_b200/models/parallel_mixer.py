"""Intra-layer hybrid: a softmax branch and a linear branch read the same
normalised input; each branch output gets its own RMSNorm; the concatenation
goes through one shared output projection:

    y = wo([norm_a(att(x)); norm_l(la(x))])

Both branches are built without their own ``wo`` (``out_proj=False``).  State
handling composes: the cache is ``{'att': ..., 'la': ...}``.

Parity: reference ``infra/components/parallel_mixer.py:37-91``.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .. import ops
from .attention import SoftmaxAttention
from .gdn import GatedDeltaNet
from .mixer import Mixer
from .norm import RMSNorm


class ParallelMixer(nn.Module, Mixer):
    def __init__(self, dim: int, *, att: SoftmaxAttention, la: GatedDeltaNet, rmsnorm_eps: float = 1e-6,
                 init_std: float = 0.02, layer_count: int | None = None):
        super().__init__()
        assert not att.out_proj and not la.out_proj, \
            "ParallelMixer owns the output projection: build branches with out_proj=False"
        assert att.in_dim == dim and la.dim == dim, "both branches read the residual width"
        self.dim = dim
        self.att = att
        self.la = la
        self.att_norm = RMSNorm(att.out_width, rmsnorm_eps)
        self.la_norm = RMSNorm(la.out_width, rmsnorm_eps)
        self.wo = nn.Linear(att.out_width + la.out_width, dim, bias=False)
        nn.init.normal_(self.wo.weight, std=init_std / math.sqrt(2 * layer_count) if layer_count else init_std)

    @property
    def gate_projections(self) -> list[nn.Parameter]:
        return self.la.gate_projections

    def _cat(self, a, b):
        return torch.cat((self.att_norm(a), self.la_norm(b)), -1)

    def forward_pre_out(self, x, is_causal: bool = True):
        return self._cat(self.att(x, is_causal), self.la(x, is_causal))

    def forward(self, x, is_causal: bool = True):
        return ops.linear(self.forward_pre_out(x, is_causal), self.wo.weight)

    def reset_cache(self, batch_size: int, max_cache_len: int):
        self.att.reset_cache(batch_size, max_cache_len)
        self.la.reset_cache(batch_size, max_cache_len)

    def load_cache(self, cache: dict, max_cache_len: int):
        self.att.load_cache(cache["att"], max_cache_len=max_cache_len)
        self.la.load_cache(cache["la"], max_cache_len=max_cache_len)

    def export_cache(self) -> dict:
        return {"att": self.att.export_cache(), "la": self.la.export_cache()}

    @torch.no_grad()
    def decode_step(self, x):
        return ops.linear(self._cat(self.att.decode_step(x), self.la.decode_step(x)), self.wo.weight)
