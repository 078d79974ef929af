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

from ._core import BF16, autocast_bf16, gemm, native


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


# ------------------------------------------------- fused projection + attention --

class _AttnLayer(torch.autograd.Function):
    """x (B, L, Din) -> the head concat (B, L, H Dv) of a softmax-attention layer
    whose q, k, v projections are one GEMM.  Column layout of the packed
    projection P: [q (H D) | k (Hk D) | v (Hk Dv)].  q and k go through the
    qk-norm + RoPE kernel (one launch over both when neither has a norm gain),
    v is read by the attention kernels straight out of P, and the backward
    writes dv, then the un-rotated dq / dk, into one gradient dP, so the input
    gradient and the three weight gradients are one GEMM each.  With RoPE and
    no qk norm the attention backward applies the rotation's transpose itself
    (tcgen05 path: sequences of 128+ tokens, equal q / v head dims)."""

    @staticmethod
    def forward(ctx, x, Wp, wq, wk, wv, qg, kg, cos, sin, meta):
        H, Hk, D, Dv, eps, causal, rotate = meta
        B, L, Din = x.shape
        Nq, Nk = H * D, Hk * D
        x2 = x.reshape(-1, Din)
        x2 = x2 if x2.is_contiguous() else x2.contiguous()
        T, NP = x2.shape[0], Wp.shape[0]
        P = torch.empty(T, NP, device=x.device, dtype=torch.bfloat16)
        gemm(x2, False, Wp, False, P)
        P4 = P.view(B, L, NP)
        C = native()
        rq = rk = None
        if not rotate:
            q, k = P4[:, :, :Nq].view(B, L, H, D), P4[:, :, Nq:Nq + Nk].view(B, L, Hk, D)
        elif qg is None and kg is None:
            qk, _ = C.qk_norm_rope_fwd(P4[:, :, :Nq + Nk].view(B, L, H + Hk, D), None, cos, sin, eps)
            q, k = qk[:, :, :H], qk[:, :, H:]
        else:
            q, rq = C.qk_norm_rope_fwd(P4[:, :, :Nq].view(B, L, H, D), qg, cos, sin, eps)
            k, rk = C.qk_norm_rope_fwd(P4[:, :, Nq:Nq + Nk].view(B, L, Hk, D), kg, cos, sin, eps)
        v = P4[:, :, Nq + Nk:].view(B, L, Hk, Dv)
        scale = 1.0 / math.sqrt(D)
        o, lse = C.attn_fwd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal, scale)
        ctx.meta = meta
        ctx.save_for_backward(x2, Wp, P, q, k, o, lse, qg, kg, cos, sin, rq, rk)
        return o.transpose(1, 2).reshape(B, L, H * Dv)

    @staticmethod
    def backward(ctx, dy):
        H, Hk, D, Dv, eps, causal, rotate = ctx.meta
        x2, Wp, P, q, k, o, lse, qg, kg, cos, sin, rq, rk = ctx.saved_tensors
        B, L = q.shape[0], q.shape[1]
        Nq, Nk = H * D, Hk * D
        T, Din = x2.shape
        NP = Wp.shape[0]
        C = native()
        dP = torch.empty(T, NP, device=x2.device, dtype=torch.bfloat16)
        P4, dP4 = P.view(B, L, NP), dP.view(B, L, NP)
        dq_slice = dP4[:, :, :Nq].view(B, L, H, D)
        dk_slice = dP4[:, :, Nq:Nq + Nk].view(B, L, Hk, D)
        dv_slice = dP4[:, :, Nq + Nk:].view(B, L, Hk, Dv)
        joint = rotate and qg is None and kg is None
        # RoPE alone: the tcgen05 backward un-rotates dq / dk itself (its dQ pass
        # and dK epilogue) and writes them straight into dP
        fused_rope = joint and cos is not None and L >= 128 and D == Dv
        if not rotate or fused_rope:
            dq, dk = dq_slice, dk_slice
        elif joint:
            dqk = torch.empty(B, L, H + Hk, D, device=x2.device, dtype=torch.bfloat16)
            dq, dk = dqk[:, :, :H], dqk[:, :, H:]
        else:
            dq = torch.empty(B, L, H, D, device=x2.device, dtype=torch.bfloat16)
            dk = torch.empty(B, L, Hk, D, device=x2.device, dtype=torch.bfloat16)
        v = P4[:, :, Nq + Nk:].view(B, L, Hk, Dv)
        dO = dy.to(torch.bfloat16).view(B, L, H, Dv).transpose(1, 2)
        C.attn_bwd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), o, lse, dO, causal, 1.0 / math.sqrt(D),
                   dq.transpose(1, 2), dk.transpose(1, 2), dv_slice.transpose(1, 2),
                   cos if fused_rope else None, sin if fused_rope else None)
        dqg = dkg = None
        if joint and not fused_rope:
            none = torch.empty(0, device=x2.device, dtype=torch.float32)
            C.qk_norm_rope_bwd(dqk, P4[:, :, :Nq + Nk].view(B, L, H + Hk, D), None, cos, sin, none,
                               dP4[:, :, :Nq + Nk].view(B, L, H + Hk, D))
        elif rotate and not joint:
            none = torch.empty(0, device=x2.device, dtype=torch.float32)
            _, g1 = C.qk_norm_rope_bwd(dq, P4[:, :, :Nq].view(B, L, H, D), qg, cos, sin,
                                       none if rq is None else rq, dq_slice)
            _, g2 = C.qk_norm_rope_bwd(dk, P4[:, :, Nq:Nq + Nk].view(B, L, Hk, D), kg, cos, sin,
                                       none if rk is None else rk, dk_slice)
            dqg = None if qg is None else g1.to(qg.dtype)
            dkg = None if kg is None else g2.to(kg.dtype)
        dx = torch.empty(T, Din, device=x2.device, dtype=torch.bfloat16)
        gemm(dP, False, Wp, True, dx)                                      # dx = dP Wp
        dWp = torch.zeros(NP, Din, device=x2.device, dtype=torch.float32)
        gemm(dP, True, x2, True, dWp, atomic=True)                         # dWp = dP^T x
        dwq, dwk, dwv = dWp.split([Nq, Nk, NP - Nq - Nk], 0)
        return dx.view(B, L, Din), None, dwq, dwk, dwv, dqg, dkg, None, None, None


def attention_layer_ok(m, x) -> bool:
    """Whether the fused projection + attention path takes this layer and input:
    CUDA, bf16 compute, no short conv or output gate, head dims 64 / 128 and
    GEMM-sized projections."""
    from .linear import gemm_ok
    if not (x.is_cuda and x.dim() == 3 and hasattr(native(), "attn_fwd")):
        return False
    if m.short_conv_size is not None or m.out_gate:
        return False
    if not (x.dtype == torch.bfloat16 or autocast_bf16()):
        return False
    if m.head_dim not in (64, 128) or m.value_head_dim not in (64, 128):
        return False
    NP = (m.head_count + m.kv_head_count) * m.head_dim + m.kv_head_count * m.value_head_dim
    return gemm_ok(x.shape[0] * x.shape[1], x.shape[2], NP)


def attention_layer(m, x, causal: bool = True):
    """Fused forward of a softmax-attention layer from its input to the head
    concat that feeds ``wo`` (q / k / v projections packed into one GEMM)."""
    L = x.shape[1]
    qg = m.q_norm.gamma if m.qk_norm else None
    kg = m.k_norm.gamma if m.qk_norm else None
    qg = None if qg is None else qg.float().contiguous()
    kg = None if kg is None else kg.float().contiguous()
    cos = sin = None
    if m.rope is not None:
        cos, sin = (t.float().contiguous() for t in m.rope.tables(L, 0))
    rotate = m.rope is not None or m.qk_norm
    eps = m.q_norm.eps if m.qk_norm else 1e-6
    Wp = BF16.get_cat([m.wq.weight, m.wk.weight, m.wv.weight])
    meta = (m.head_count, m.kv_head_count, m.head_dim, m.value_head_dim, float(eps), bool(causal), rotate)
    return _AttnLayer.apply(x.to(torch.bfloat16), Wp, m.wq.weight, m.wk.weight, m.wv.weight, qg, kg, cos, sin, meta)
