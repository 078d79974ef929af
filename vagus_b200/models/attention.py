"""Multi-head softmax attention: RoPE or NoPE, GQA, widened V, optional short
conv on q/k/v, per-head qk RMSNorm before RoPE, optional sigmoid output gate.

On CUDA the training forward runs the fused qk-norm + RoPE kernel and the
sm_100a flash-attention kernels (``vagus_b200.ops.attention``); decode with a
KV cache uses the same kernels with a lower-right causal mask (query i sits at
absolute position offset + i).  ``max_attn_logit`` is a probe (fp32, full
score matrix, small inputs only).

Parity: reference ``infra/components/attention.py:16-382``.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .. import ops
from ..utils import infer_device, infer_dtype
from .conv import ShortConv
from .mixer import Mixer
from .norm import RMSNorm
from .rope import RoPE


class SoftmaxAttention(nn.Module, Mixer):
    def __init__(self, dim: int, head_count: int, kv_head_count: int | None, v_dim_mult: int,
                 short_conv_size: int | None = None, qk_norm: bool = False, *, rope: RoPE | None,
                 init_std: float = 0.02, layer_count: int | None = None, in_dim: int | None = None,
                 out_proj: bool = True, out_gate: bool = False):
        super().__init__()
        if kv_head_count is None:
            kv_head_count = head_count
        assert dim % head_count == 0 and head_count % kv_head_count == 0 and v_dim_mult > 0
        assert rope is None or rope.head_dim == dim // head_count
        self.dim = dim
        self.in_dim = in_dim or dim
        self.out_proj = out_proj
        self.out_gate = out_gate
        self.v_dim_mult = v_dim_mult
        self.out_width = dim * v_dim_mult
        self.head_count = head_count
        self.kv_head_count = kv_head_count
        self.short_conv_size = short_conv_size
        self.qk_norm = qk_norm
        self.rope = rope
        Dh = dim // head_count
        self.wq = nn.Linear(self.in_dim, dim, bias=False)
        self.wk = nn.Linear(self.in_dim, Dh * kv_head_count, bias=False)
        self.wv = nn.Linear(self.in_dim, Dh * kv_head_count * v_dim_mult, bias=False)
        if out_proj:
            self.wo = nn.Linear(self.out_width, dim, bias=False)
        if out_gate:
            self.wg = nn.Linear(self.in_dim, self.out_width, bias=False)
        if short_conv_size is not None:
            self.conv_q = ShortConv(dim, short_conv_size)
            self.conv_k = ShortConv(Dh * kv_head_count, short_conv_size)
            self.conv_v = ShortConv(Dh * kv_head_count * v_dim_mult, short_conv_size)
        if qk_norm:
            self.q_norm = RMSNorm(Dh)
            self.k_norm = RMSNorm(Dh)
        for lin in (self.wq, self.wk, self.wv):
            nn.init.normal_(lin.weight, std=init_std)
        if out_gate:
            nn.init.normal_(self.wg.weight, std=init_std)
        if out_proj:
            nn.init.normal_(self.wo.weight, std=init_std / math.sqrt(2 * layer_count) if layer_count else init_std)
        self.cache_len = 0
        self.register_buffer("k_cache", torch.zeros(0, 0, 0, 0), persistent=False)
        self.register_buffer("v_cache", torch.zeros(0, 0, 0, 0), persistent=False)
        if short_conv_size is not None:
            self.register_buffer("qp_cache", torch.zeros(0, short_conv_size, dim), persistent=False)
            self.register_buffer("kp_cache", torch.zeros(0, short_conv_size, Dh * kv_head_count), persistent=False)
            self.register_buffer("vp_cache", torch.zeros(0, short_conv_size, Dh * kv_head_count * v_dim_mult),
                                 persistent=False)

    @property
    def head_dim(self) -> int:
        return self.dim // self.head_count

    @property
    def value_head_dim(self) -> int:
        return self.dim * self.v_dim_mult // self.head_count

    def _qk(self, qp, kp, offset: int):
        """(B, L, width) projections -> normalised, rotated (B, H, L, Dh) heads."""
        B, L = qp.shape[0], qp.shape[1]
        H, Hk, Dh = self.head_count, self.kv_head_count, self.head_dim
        q = qp.reshape(B, L, H, Dh)
        k = kp.reshape(B, L, Hk, Dh)
        qn = self.q_norm.gamma if self.qk_norm else None
        kn = self.k_norm.gamma if self.qk_norm else None
        eps = self.q_norm.eps if self.qk_norm else 1e-6
        tables = self.rope.tables(L, offset) if self.rope is not None else None
        q = ops.qk_norm_rope(q, qn, tables, eps)
        k = ops.qk_norm_rope(k, kn, tables, eps)
        return q.transpose(1, 2), k.transpose(1, 2)

    def forward(self, x, is_causal: bool = True):
        out = self.forward_pre_out(x, is_causal)
        return ops.linear(out, self.wo.weight) if self.out_proj else out

    def forward_pre_out(self, x, is_causal: bool = True):
        """The (gated) head concat that feeds ``wo``.  On CUDA in bf16 without
        short conv or output gate the q / k / v projections run as one packed
        GEMM inside ``ops.attention_layer``."""
        if ops.attention_layer_ok(self, x):
            return ops.attention_layer(self, x, is_causal)
        B, L = x.shape[0], x.shape[1]
        qp, kp, vp = ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight), ops.linear(x, self.wv.weight)
        if self.short_conv_size is not None:
            qp, kp, vp = self.conv_q(qp), self.conv_k(kp), self.conv_v(vp)
        q, k = self._qk(qp, kp, 0)
        v = vp.reshape(B, L, self.kv_head_count, self.value_head_dim).transpose(1, 2)
        out = ops.attention(q, k, v, causal=is_causal)                 # (B, H, L, Dvh)
        out = out.transpose(1, 2).reshape(B, L, -1)
        if self.out_gate:
            out = ops.sigmoid_gate(out, ops.linear(x, self.wg.weight))
        return out

    @torch.no_grad()
    def max_attn_logit(self, x) -> torch.Tensor:
        """Max causal pre-softmax logit (fp32, materialised scores)."""
        B, L = x.shape[0], x.shape[1]
        qp, kp = ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight)
        if self.short_conv_size is not None:
            qp, kp = self.conv_q(qp), self.conv_k(kp)
        q, k = self._qk(qp, kp, 0)
        if self.kv_head_count != self.head_count:
            k = k.repeat_interleave(self.head_count // self.kv_head_count, dim=1)
        scores = q.float() @ k.float().transpose(-1, -2) / math.sqrt(self.head_dim)
        causal = torch.ones(L, L, dtype=torch.bool, device=x.device).tril()
        return scores.masked_fill(~causal, float("-inf")).amax()

    # --- streaming ---------------------------------------------------------

    def reset_cache(self, batch_size: int, max_cache_len: int):
        device, dtype = infer_device(self), infer_dtype(self)
        Hk, Dh, Dvh = self.kv_head_count, self.head_dim, self.value_head_dim
        self.cache_len = 0
        self.k_cache = torch.zeros(batch_size, Hk, max_cache_len, Dh, device=device, dtype=dtype)
        self.v_cache = torch.zeros(batch_size, Hk, max_cache_len, Dvh, device=device, dtype=dtype)
        if self.short_conv_size is not None:
            K = self.short_conv_size
            self.qp_cache = torch.zeros(batch_size, K, self.dim, device=device, dtype=dtype)
            self.kp_cache = torch.zeros(batch_size, K, Dh * Hk, device=device, dtype=dtype)
            self.vp_cache = torch.zeros(batch_size, K, Dvh * Hk, device=device, dtype=dtype)
        if self.rope is not None:
            self.rope.prepare_m(max_cache_len)

    def load_cache(self, cache: dict, max_cache_len: int):
        prefix = cache["k_cache"].shape[2]
        if prefix > max_cache_len:
            raise ValueError("The cache length already exceeds the given max_cache_len.")
        self.reset_cache(cache["k_cache"].shape[0], max_cache_len)
        self.cache_len = prefix
        self.k_cache[:, :, :prefix].copy_(cache["k_cache"])
        self.v_cache[:, :, :prefix].copy_(cache["v_cache"])
        if self.short_conv_size is not None:
            self.qp_cache.copy_(cache["qp_cache"])
            self.kp_cache.copy_(cache["kp_cache"])
            self.vp_cache.copy_(cache["vp_cache"])

    def export_cache(self) -> dict:
        out = {"k_cache": self.k_cache[:, :, :self.cache_len].clone(),
               "v_cache": self.v_cache[:, :, :self.cache_len].clone()}
        if self.short_conv_size is not None:
            out.update(qp_cache=self.qp_cache.clone(), kp_cache=self.kp_cache.clone(),
                       vp_cache=self.vp_cache.clone())
        return out

    @torch.no_grad()
    def decode_step(self, x):
        """Streaming continuation against the KV cache (keys cached post-RoPE)."""
        B, L = x.shape[0], x.shape[1]
        assert x.dtype == self.k_cache.dtype and x.device == self.k_cache.device
        assert self.k_cache.shape[2] > 0, "No cache allocated. Call reset_cache or load_cache first."
        assert B == self.k_cache.shape[0], "The input batch_size does not match with the cache."
        offset = self.cache_len
        T = offset + L
        assert T <= self.k_cache.shape[2], "Cache overflow. Allocate with a larger max_cache_len."
        qp, kp, vp = ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight), ops.linear(x, self.wv.weight)
        if self.short_conv_size is not None:
            K = self.short_conv_size
            qp = torch.cat([self.qp_cache, qp], 1)
            kp = torch.cat([self.kp_cache, kp], 1)
            vp = torch.cat([self.vp_cache, vp], 1)
            self.qp_cache.copy_(qp[:, -K:])
            self.kp_cache.copy_(kp[:, -K:])
            self.vp_cache.copy_(vp[:, -K:])
            qp = self.conv_q.direct_conv(qp)[:, -L:]
            kp = self.conv_k.direct_conv(kp)[:, -L:]
            vp = self.conv_v.direct_conv(vp)[:, -L:]
        q, k = self._qk(qp, kp, offset)
        v = vp.reshape(B, L, self.kv_head_count, self.value_head_dim).transpose(1, 2)
        self.k_cache[:, :, offset:T].copy_(k)
        self.v_cache[:, :, offset:T].copy_(v)
        self.cache_len = T
        out = ops.attention(q, self.k_cache[:, :, :T], self.v_cache[:, :, :T], causal=True)
        out = out.transpose(1, 2).reshape(B, L, -1)
        if self.out_gate:
            out = ops.sigmoid_gate(out, ops.linear(x, self.wg.weight))
        return ops.linear(out, self.wo.weight) if self.out_proj else out
