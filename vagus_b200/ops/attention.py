"""Softmax attention: q (B, H, Lq, D), k (B, Hk, Lk, D), v (B, Hk, Lk, Dv).

``causal=True`` aligns the mask lower-right: query i sits at absolute
position Lk - Lq + i (training Lq == Lk is the ordinary causal mask; a
single decode query sees the whole prefix).  GQA when Hk < H.  Scale
1/sqrt(D).  CUDA runs the sm_100a flash-attention kernels (attention.cu).
"""

from __future__ import annotations

import math

import torch
from torch.nn import functional as F
from torch.nn.attention.bias import causal_lower_right

from ._core import native


def attention_ref(q, k, v, causal: bool = True):
    H, Hk = q.shape[1], k.shape[1]
    Lq, Lk = q.shape[2], k.shape[2]
    gqa = H != Hk
    if causal and Lq == Lk:
        return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=gqa)
    if causal and Lq > 1:
        return F.scaled_dot_product_attention(q, k, v, attn_mask=causal_lower_right(Lq, Lk), enable_gqa=gqa)
    return F.scaled_dot_product_attention(q, k, v, enable_gqa=gqa)


class _Attn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal):
        o, lse = native().attn_fwd(q, k, v, causal, 1.0 / math.sqrt(q.shape[-1]))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        # dO arrives in o's (token-major) layout from the head concat; the
        # gradients leave in the layouts of q, k, v: no transposing copies
        dq, dk, dv = native().attn_bwd(q, k, v, o, lse, do, ctx.causal, 1.0 / math.sqrt(q.shape[-1]))
        return dq, dk, dv, None


def attention(q, k, v, causal: bool = True):
    if q.is_cuda and q.dtype == torch.bfloat16 and hasattr(native(), "attn_fwd") \
            and q.shape[-1] in (64, 128) and v.shape[-1] in (64, 128):
        return _Attn.apply(q, k, v, bool(causal))
    return attention_ref(q, k, v, causal)
