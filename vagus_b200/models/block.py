"""Pre-norm residual block shared by every model:

    x = x + mixer(RMSNorm(x));   x = x + FFN(RMSNorm(x))

The mixer is injected (any ``Mixer``) and kept under the attribute ``att``.
On CUDA the two residual adds are fused into the epilogues of the output GEMMs
(``wo`` and ``ffn.l2``): the GEMM kernel reads the fp32 residual and writes
residual + product, so the residual stream makes one round trip per sub-layer.
In the backward the residual gradient is added inside the norm kernel
(``ops.rmsnorm_pass``), which also hands the output GEMM a bf16 copy.

Parity: reference ``infra/components/block.py:19-91``.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .. import ops
from .cache import WithCache
from .ffn import FFN
from .mixer import Mixer, missing_mixer
from .norm import RMSNorm


class Block(nn.Module, WithCache):
    def __init__(self, dim: int, ffn_hidden_dim: int | None = None, rmsnorm_eps: float = 1e-6, *,
                 mixer: Mixer, layer_count: int | None):
        super().__init__()
        missing = missing_mixer(mixer)
        if missing:
            raise TypeError(f"{type(mixer).__name__} is not a Mixer: missing {missing}")
        # Llama SwiGLU sizing: 8/3 dim rounded up to a multiple of 256
        ffn_hidden_dim = ffn_hidden_dim or math.ceil(int(8 * dim / 3) / 256) * 256
        self.rmsnorm1 = RMSNorm(dim, rmsnorm_eps)
        self.att: Mixer = mixer
        self.rmsnorm2 = RMSNorm(dim, rmsnorm_eps)
        self.ffn = FFN(dim=dim, hidden_dim=ffn_hidden_dim, init_std=0.02, layer_count=layer_count)

    def _fused(self, x: torch.Tensor) -> bool:
        return ops.kernels_active(x) and hasattr(self.att, "forward_pre_out") and hasattr(self.att, "wo")

    def forward(self, x, is_causal: bool = True):
        if self._fused(x):
            h, x = ops.rmsnorm_pass(x, self.rmsnorm1.gamma, self.rmsnorm1.eps)
            x = ops.linear_residual(x, self.att.forward_pre_out(h, is_causal), self.att.wo.weight)
            h, x = ops.rmsnorm_pass(x, self.rmsnorm2.gamma, self.rmsnorm2.eps)
            return ops.linear_residual(x, self.ffn.hidden(h), self.ffn.l2.weight)
        x = x + self.att(self.rmsnorm1(x), is_causal)
        return x + self.ffn(self.rmsnorm2(x))

    def reset_cache(self, batch_size: int, max_cache_len: int):
        self.att.reset_cache(batch_size, max_cache_len)

    def load_cache(self, cache: dict, max_cache_len: int):
        self.att.load_cache(cache["att"], max_cache_len=max_cache_len)

    def export_cache(self) -> dict:
        return {"att": self.att.export_cache()}

    @torch.no_grad()
    def decode_step(self, x):
        x = x + self.att.decode_step(self.rmsnorm1(x))
        return x + self.ffn(self.rmsnorm2(x))
