"""Gated delta-rule ops on CUDA.

``gdr_chunk``   the chunked scan (scalar gate): the intra-chunk kernel
                (gdr_intra.cu) builds W, U, Qh, Kt, A and gC per 64-token
                chunk, the recurrence kernel (gdr.cu) runs the inter-chunk
                state scan; backward runs the reverse scan and then the
                intra-chunk derivative kernel.  ``_intra`` below is the same
                intra-chunk algebra in PyTorch (the tests' oracle).
``gdr_decode``  single-token recurrent step (state updated in place).
``gdn_mixer``   one Gated DeltaNet layer up to the input of ``wo`` as a single
                autograd node: packed q|k|v|g GEMM, packed a|b GEMM, fused
                conv+SiLU+L2norm, gate activation, chunk scan, RMSNorm*SiLU
                gate; the backward writes every gradient of the packed
                projection into one buffer and runs one dgrad and one wgrad
                GEMM for it.
"""

from __future__ import annotations

import torch

from ._core import BF16, as_bf16_2d, gemm, native

CHUNK = 64


def _intra(q, k, v, g, beta, scale: float):
    """Per-chunk operands of the recurrence, fp32.  q, k (B, L, H, dk); v (B,
    L, H, dv); g, beta (B, L, H); L a multiple of the chunk size.
    Returns W, Qh, Kt (B, H, N, C, dk), A (B, H, N, C, C), U (B, H, N, C, dv),
    gC (B, H, N)."""
    B, L, H, dk = q.shape
    C = CHUNK
    N = L // C

    def ch(t):
        return t.float().view(B, N, C, H, t.shape[-1]).permute(0, 3, 1, 2, 4)

    Q, K, V = ch(q), ch(k), ch(v)
    gam = g.float().view(B, N, C, H).permute(0, 3, 1, 2).cumsum(-1)            # (B, H, N, C)
    b = beta.float().view(B, N, C, H).permute(0, 3, 1, 2)
    causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    D = (gam[..., :, None] - gam[..., None, :]).masked_fill(~causal, float("-inf")).exp()
    G = gam.exp()
    gC = G[..., -1]
    Akk = (b[..., :, None] * (K @ K.transpose(-1, -2)) * D).tril(-1)
    Tm = Akk + torch.eye(C, device=q.device, dtype=Akk.dtype)
    W = torch.linalg.solve_triangular(Tm, (b * G)[..., None] * K, upper=False, unitriangular=True)
    U = torch.linalg.solve_triangular(Tm, b[..., None] * V, upper=False, unitriangular=True)
    Qh = (G * scale)[..., None] * Q
    Kt = (gam[..., -1:] - gam).exp()[..., None] * K
    A = (Q @ K.transpose(-1, -2)) * D * scale
    return W, Qh, Kt, A, U, gC


def _flat(t):
    B, H = t.shape[0], t.shape[1]
    return t.reshape(B * H, *t.shape[2:])


def _gdr_fwd(q, k, v, g, beta, S0, scale):
    """Forward of the chunk scan; returns (o, S_final, saved) with ``saved``
    the tensors the backward needs."""
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    N = L // CHUNK
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    g, beta = g.float().contiguous(), beta.float().contiguous()
    W, Qh, Kt, A, U, gCf = native().gdr_intra_fwd(q, k, v, g, beta, scale)
    ops16 = [W, Qh, Kt, A, U]
    S0f = None if S0 is None else S0.float().reshape(B * H, dk, dv).contiguous()
    o, Vp, states, S_out = native().gdr_rec_fwd(*ops16, gCf, S0f, True, H)     # o token-major (B, L, H, dv)
    saved = (q, k, v, g, beta, ops16[0], ops16[1], ops16[2], ops16[3], Vp, gCf, states)
    return o, S_out.view(B, H, dk, dv), saved


def _gdr_bwd(saved, do, dS, scale, need_dS0):
    """Gradients (dq, dk, dv, dg, dbeta, dS0) of the chunk scan."""
    q, k, v, g, beta, W16, Qh16, Kt16, A16, Vp, gCf, states = saved
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    N = L // CHUNK
    dO = do.to(torch.bfloat16).reshape(B, L, H, dv).contiguous()          # token-major, as the kernels read it
    dSf = None if dS is None else dS.float().reshape(B * H, dk, dv).contiguous()
    dW, dQh, dKt, dA, dU, dgC, dS0 = native().gdr_rec_bwd(W16, Qh16, Kt16, A16, Vp, gCf, states,
                                                          dO, dSf, need_dS0)
    gq, gk, gv, gg, gb = native().gdr_intra_bwd(q, k, v, g, beta, dW, dQh, dKt, dA, dU, dgC, scale)
    return gq, gk, gv, gg, gb, (dS0.view(B, H, dk, dv) if need_dS0 else None)


class _GDRChunk(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, S0, scale):
        o, S, saved = _gdr_fwd(q, k, v, g, beta, S0, scale)
        ctx.save_for_backward(*saved)
        ctx.scale = scale
        ctx.has_S0 = S0 is not None
        return o, S

    @staticmethod
    def backward(ctx, do, dS):
        gq, gk, gv, gg, gb, dS0 = _gdr_bwd(ctx.saved_tensors, do, dS, ctx.scale, ctx.has_S0)
        return gq, gk, gv, gg, gb, dS0, None


def gdr_chunk(q, k, v, g, beta, S0, *, scale: float, chunk_size: int = 64):
    """Chunked gated delta rule with a scalar gate on CUDA (bf16 q/k/v).
    Returns (o (B, L, H, dv) bf16, S (B, H, dk, dv) fp32)."""
    assert chunk_size == CHUNK, "the sm_100a recurrence runs 64-token chunks"
    B, L, H, dk = q.shape
    pad = (-L) % CHUNK
    if pad:
        pz = lambda t: torch.nn.functional.pad(t, [0, 0] * (t.dim() - 2) + [0, pad])   # noqa: E731
        q, k, v, g, beta = pz(q), pz(k), pz(v), pz(g), pz(beta)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    o, S = _GDRChunk.apply(q, k, v, g.float(), beta.float(), S0, scale)
    return (o[:, :L] if pad else o), S


def gdr_decode(q, k, v, g, beta, S, *, scale: float):
    """One recurrent step.  q, k (B, 1, H, dk); v (B, 1, H, dv); g, beta
    (B, 1, H); S (B, H, dk, dv) fp32.  Returns (o (B, 1, H, dv), S')."""
    B, _, H, dk = q.shape
    dv = v.shape[-1]
    S2 = S.float().contiguous().clone()
    o = native().gdr_decode(q.reshape(B * H, dk).to(torch.bfloat16), k.reshape(B * H, dk).to(torch.bfloat16),
                            v.reshape(B * H, dv).to(torch.bfloat16), g.reshape(B * H).float(),
                            beta.reshape(B * H).float(), S2.view(B * H, dk, dv), scale)
    return o.view(B, 1, H, dv).to(q.dtype), S2


# ------------------------------------------------- short conv as an op --

class _ConvSilu(torch.autograd.Function):
    """Causal depthwise conv + SiLU (+ per-head L2 norm) on the conv kernels,
    for layers outside the fused mixer (the per-channel-gate path)."""

    @staticmethod
    def forward(ctx, x, w, head_dim: int, l2norm: bool):
        x = x.to(torch.bfloat16).contiguous()
        wf = w.float().contiguous()
        y, rn = native().conv_silu_fwd(x, wf, head_dim, l2norm)
        ctx.save_for_backward(x, wf, rn)
        ctx.cfg = (head_dim, l2norm, w.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, wf, rn = ctx.saved_tensors
        head_dim, l2norm, wdt = ctx.cfg
        dx = torch.empty_like(x)
        dw = torch.zeros(wf.numel(), device=x.device, dtype=torch.float32)
        native().conv_silu_bwd(dy.to(torch.bfloat16).contiguous(), x, wf, rn, dx, dw, head_dim, l2norm)
        return dx, dw.view(wf.shape).to(wdt), None, None


def conv_silu(x, w, head_dim: int, l2norm: bool):
    """x (B, L, D) -> SiLU(causal depthwise conv(x, w)) (B, L, D) bf16, each
    head_dim group L2-normalised when ``l2norm``; w (D, 1, K)."""
    return _ConvSilu.apply(x, w, head_dim, l2norm)


# ------------------------------------------------------------- fused layer --

def _packed_weight(m):
    """bf16 rows [wq; wk; wv; wg; wa; wb; 0-pad] of one layer: every input
    projection of the layer is one GEMM.  The zero rows pad the count to a
    multiple of 64 (the weight-gradient GEMM reads it in 64-row blocks)."""
    ws = [m.wq.weight, m.wk.weight, m.wv.weight, m.wg.weight, m.wa.weight, m.wb.weight]
    n = sum(w.shape[0] for w in ws)
    pad = (-n) % 64
    key = ("gdn_pad", pad, m.dim)
    zeros = _PAD.get(key)
    if zeros is None or zeros.device != ws[0].device:
        zeros = torch.zeros(pad, m.dim, device=ws[0].device, dtype=torch.float32)
        _PAD[key] = zeros
    return BF16.get_cat(ws + [zeros]), n


_PAD: dict = {}


class _GDNMixer(torch.autograd.Function):
    """h (B, L, D) bf16 -> the gated normalised head concat (B, L, H dv).
    Column layout of the packed projection P: [q | k | v | g | a | b | pad]."""

    @staticmethod
    def forward(ctx, h, Wp, wq, wk, wv, wg, wa, wb, A_log, dt_bias, cq, ck, cv, gamma, meta):
        H, dk, dv, eps, scale = meta
        B, L, Dm = h.shape
        Hk, Hv = H * dk, H * dv
        h2 = as_bf16_2d(h)
        T = h2.shape[0]
        NP = Wp.shape[0]
        P = torch.empty(T, NP, device=h.device, dtype=torch.bfloat16)
        gemm(h2, False, Wp, False, P)
        P3 = P.view(B, L, NP)
        oa = 2 * Hk + 2 * Hv                                                  # a|b column offset
        C = native()
        # the kernels take fp32 taps (a no-op for fp32 masters; bf16 under FSDP mixed precision)
        cq, ck, cv = cq.float().contiguous(), ck.float().contiguous(), cv.float().contiguous()
        q, rq = C.conv_silu_fwd(P3[:, :, :Hk], cq, dk, True)
        k, rk = C.conv_silu_fwd(P3[:, :, Hk:2 * Hk], ck, dk, True)
        v, _ = C.conv_silu_fwd(P3[:, :, 2 * Hk:2 * Hk + Hv], cv, dv, False)
        g, beta = C.gdn_gates_fwd(P[:, oa:oa + 2 * H], A_log.float().contiguous(), dt_bias.float().contiguous(), H)
        o, _S, gsaved = _gdr_fwd(q.view(B, L, H, dk), k.view(B, L, H, dk), v.view(B, L, H, dv),
                                 g.view(B, L, H), beta.view(B, L, H), None, scale)
        o = o.contiguous()
        y, rstd = C.rmsnorm_gated_fwd(o.view(T, H, dv), P[:, 2 * Hk + Hv:oa], gamma.float().contiguous(), eps, H)
        ctx.dims = (B, L, Dm, H, dk, dv, NP)
        ctx.scale = scale
        ctx.save_for_backward(h2, Wp, P, rq, rk, o, rstd, A_log, dt_bias, cq, ck, cv, gamma, *gsaved)
        return y.view(B, L, Hv)

    @staticmethod
    def backward(ctx, dy):
        B, L, Dm, H, dk, dv, NP = ctx.dims
        Hk, Hv = H * dk, H * dv
        oa = 2 * Hk + 2 * Hv
        sv = ctx.saved_tensors
        h2, Wp, P, rq, rk, o, rstd, A_log, dt_bias, cq, ck, cv, gamma = sv[:13]
        gsaved = sv[13:]
        T = h2.shape[0]
        C = native()
        dP = torch.empty(T, NP, device=h2.device, dtype=torch.bfloat16)
        if NP > oa + 2 * H:
            dP[:, oa + 2 * H:].zero_()
        do, dgamma = C.rmsnorm_gated_bwd(dy.reshape(T, Hv).to(torch.bfloat16), o.view(T, H, dv),
                                         P[:, 2 * Hk + Hv:oa], gamma.float().contiguous(), rstd,
                                         dP[:, 2 * Hk + Hv:oa], H)
        gq, gk, gv, gg, gb, _ = _gdr_bwd(gsaved, do.view(B, L, H, dv), None, ctx.scale, False)
        dA_log, ddt = C.gdn_gates_bwd(gg.reshape(T, H), gb.reshape(T, H), P[:, oa:oa + 2 * H],
                                      A_log.float().contiguous(), dt_bias.float().contiguous(), H,
                                      dP[:, oa:oa + 2 * H])
        P3, dP3 = P.view(B, L, NP), dP.view(B, L, NP)
        dcq = torch.zeros(cq.numel(), device=h2.device, dtype=torch.float32)
        dck = torch.zeros(ck.numel(), device=h2.device, dtype=torch.float32)
        dcv = torch.zeros(cv.numel(), device=h2.device, dtype=torch.float32)
        C.conv_silu_bwd(gq.reshape(B, L, Hk), P3[:, :, :Hk], cq, rq, dP3[:, :, :Hk], dcq, dk, True)
        C.conv_silu_bwd(gk.reshape(B, L, Hk), P3[:, :, Hk:2 * Hk], ck, rk, dP3[:, :, Hk:2 * Hk], dck, dk, True)
        C.conv_silu_bwd(gv.reshape(B, L, Hv), P3[:, :, 2 * Hk:2 * Hk + Hv], cv, rq, dP3[:, :, 2 * Hk:2 * Hk + Hv],
                        dcv, dv, False)
        dh = torch.empty(T, Dm, device=h2.device, dtype=torch.bfloat16)
        gemm(dP, False, Wp, True, dh)                                          # dh = dP Wp
        dWp = torch.zeros(NP, Dm, device=h2.device, dtype=torch.float32)
        gemm(dP, True, h2, True, dWp, atomic=True)                             # dWp = dP^T h
        dwq, dwk, dwv, dwg, dwa, dwb = dWp[:oa + 2 * H].split([Hk, Hk, Hv, Hv, H, H], 0)
        return (dh.view(B, L, Dm), None, dwq, dwk, dwv, dwg, dwa, dwb, dA_log, ddt, dcq.view_as(cq),
                dck.view_as(ck), dcv.view_as(cv), dgamma, None)


def gdn_mixer(m, x):
    """Fused forward of a GatedDeltaNet layer (scalar gate, delta rule, short
    conv) up to the input of ``wo``."""
    B, L, _ = x.shape
    meta = (m.head_count, m.key_head_dim, m.value_head_dim, m.o_norm.eps, m.scale)
    pad = (-L) % CHUNK
    if pad:
        x = torch.nn.functional.pad(x, (0, 0, 0, pad))
    Wp, _ = _packed_weight(m)
    y = _GDNMixer.apply(x.to(torch.bfloat16), Wp, m.wq.weight, m.wk.weight, m.wv.weight, m.wg.weight,
                        m.wa.weight, m.wb.weight, m.A_log, m.dt_bias, m.conv_q.conv.weight, m.conv_k.conv.weight,
                        m.conv_v.conv.weight, m.o_norm.gamma, meta)
    return y[:, :L] if pad else y
