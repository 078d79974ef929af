"""Chunked delta rule with a per-channel (Kimi-delta, KDA) gate on CUDA.

For key head dim 128 (value head dim 128 or 256) with the delta rule the
whole layer runs on our kernels (``_KDAFused``): the intra-chunk stage in
``csrc/kda_intra.cu`` (per-channel cumulative decay, gated products on the
tensor cores across 16-token blocks and elementwise inside them, the WY
transform) and the state recurrence on the GDR recurrence kernels
(``csrc/gdr.cu``: tcgen05 forward scan, chunk-parallel output and gradient
kernels), whose chunk decay gC is a per-key-channel vector.  Other variants
(no delta rule, an explicit write vector, other head dims) run the intra
stage below in torch, chunk-parallel over the whole sequence (fp32), on the
same recurrence kernels.

Per chunk of C = 64 tokens with in-chunk cumulative log decay g_i (a dk
vector, non-increasing in i), gated inner products
<x_i, y_j>_g = sum_c x_ic y_jc exp(g_ic - g_jc) (i >= j) give
    M = tril(diag(beta) <K, K>_g, -1),  T = (I + M)^-1
    W = T diag(beta) (K o e^g),  U = T diag(beta) V
    Qh = scale Q o e^g,  Kt = K o e^(g_last - g),  A = scale tril(<Q, K>_g)
    gamma = e^(g_last)
and the recurrence V' = U - W S, O = Qh S + A V', S <- diag(gamma) S + Kt^T V'.
On CUDA the gated products come from ``csrc/kda.cu`` (the pairwise decay
elementwise, one exponential per (i, j, channel) shared by both products);
the torch fallback forms them on 16-row sub-chunks: across sub-chunks the
decay factorises through the sub-chunk boundaries with every exponent <= 0
(no overflow for fast channels), inside a sub-chunk the 16 x 16 x dk decay
is taken elementwise.

Parity: the reference runs fla's ``chunk_kda`` Triton kernels
(``infra/components/linear_attention.py``); the math is the chunk form of
its recurrence (``models/scans.py`` ``chunk_scan_vec`` is the oracle).
"""

from __future__ import annotations

import torch

from ._core import BF16, as_bf16_2d, gemm, native

CHUNK = 64
SUB = 16


def _gated(X: torch.Tensor, Y: torch.Tensor, g: torch.Tensor, strict: bool) -> torch.Tensor:
    """sum_c X_ic Y_jc exp(g_ic - g_jc) for j <= i (j < i when strict), zero
    above; X, Y, g (..., C, dk) fp32 -> (..., C, C)."""
    *lead, C, dk = X.shape
    nb = C // SUB
    Xb, Yb, gb = (t.reshape(*lead, nb, SUB, dk) for t in (X, Y, g))
    first = gb[..., :, :1, :]                                   # (..., nb, 1, dk): g at each sub-chunk start
    # across sub-chunks (block I > J): exp(g_i - g_j) = exp(g_i - f_I) exp(f_I - f_{J+1}) exp(f_{J+1} - g_j)
    Xs = Xb * (gb - first).exp()                                # rows scaled to their sub-chunk start
    nxt = torch.cat([first[..., 1:, :, :], gb[..., -1:, -1:, :]], dim=-3)   # f_{J+1} (last block: unused)
    Ys = Yb * (nxt - gb).exp()                                  # columns scaled to the next sub-chunk start
    f = first.squeeze(-2)                                       # (..., nb, dk)
    fn = nxt.squeeze(-2)
    Dm = (f[..., :, None, :] - fn[..., None, :, :])             # (..., I, J, dk): f_I - f_{J+1}
    low = torch.ones(nb, nb, dtype=torch.bool, device=X.device).tril(-1)
    Dm = Dm.masked_fill(~low[..., None], float("-inf")).exp()   # zero unless J < I
    out = torch.einsum("...isc,...ijc,...jtc->...isjt", Xs, Dm, Ys)          # (..., I, 16, J, 16)
    # inside a sub-chunk: the decay elementwise
    E = gb[..., :, :, None, :] - gb[..., :, None, :, :]          # (..., nb, 16, 16, dk)
    tri = torch.ones(SUB, SUB, dtype=torch.bool, device=X.device).tril(-1 if strict else 0)
    E = E.masked_fill(~tri[..., None], float("-inf")).exp()
    diag = torch.einsum("...bic,...bijc,...bjc->...bij", Xb, E, Yb)           # (..., nb, 16, 16)
    eye = torch.eye(nb, dtype=X.dtype, device=X.device)
    out = out + diag[..., :, :, None, :] * eye[:, None, :, None]
    return out.reshape(*lead, C, C)


class _GatedProducts(torch.autograd.Function):
    """(Aqk causal, Akk strict) of every chunk on the CUDA kernels (kda.cu)."""

    @staticmethod
    def forward(ctx, Q, K, gam):
        Q, K, gam = Q.contiguous(), K.contiguous(), gam.contiguous()
        Aqk, Akk = native().kda_gated_fwd(Q, K, gam)
        ctx.save_for_backward(Q, K, gam)
        return Aqk, Akk

    @staticmethod
    def backward(ctx, dAqk, dAkk):
        Q, K, gam = ctx.saved_tensors
        zeros = lambda: torch.zeros(*Q.shape[:-1], Q.shape[-2], device=Q.device)   # noqa: E731
        dQ, dK, dG = native().kda_gated_bwd(Q, K, gam, dAqk if dAqk is not None else zeros(),
                                            dAkk if dAkk is not None else zeros())
        return dQ, dK, dG


def kda_intra(q, k, v, g, beta, scale: float, delta: bool = True, w=None):
    """(W, Qh, Kt, A, U, gamma) of every chunk, fp32, (B, H, N, C, .) layout;
    q, k (B, L, H, dk), v (B, L, H, dv), g (B, L, H, dk) log decay, beta (B, L, H).
    Without the delta rule (gated linear attention: S <- diag(gamma) S + Kt^T V)
    W is zero and U = V, so the same recurrence kernels apply.  With an
    explicit write vector w (B, L, H, dk) (the asymmetric write
    S <- S + w (v - S^T k)^T, beta unused) the read key k and the write w
    take separate slots: M = tril(<K, Wr>_g, -1), T = (I + M)^-1, U = T V,
    W = T (K o e^g), A = scale tril(<Q, Wr>_g), Kt = Wr o e^(g_last - g)."""
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    N = L // CHUNK
    to_c = lambda t, d: t.float().reshape(B, N, CHUNK, H, d).permute(0, 3, 1, 2, 4)   # noqa: E731
    Q, K, V = to_c(q, dk), to_c(k, dk), to_c(v, dv)
    gam = to_c(g, dk).cumsum(3)                                  # (B, H, N, C, dk)
    if w is not None:
        # gated products with the write vectors in the column slot (torch,
        # chunk-parallel; the CUDA products share one column operand)
        Wr = to_c(w, dk)
        Aqw, Akw = _gated(Q, Wr, gam, strict=False), _gated(K, Wr, gam, strict=True)
        G = gam.exp()
        Tm = Akw + torch.eye(CHUNK, device=q.device, dtype=Akw.dtype)
        eye = torch.eye(CHUNK, device=q.device, dtype=Akw.dtype).expand_as(Tm)
        T = torch.linalg.solve_triangular(Tm, eye, upper=False, unitriangular=True)
        WU = T @ torch.cat([K * G, V], dim=-1)
        return (WU[..., :dk], Q * G * scale, Wr * (gam[..., -1:, :] - gam).exp(), Aqw * scale, WU[..., dk:],
                G[..., -1, :])
    if q.is_cuda:
        Aqk, Akk = _GatedProducts.apply(Q, K, gam)
    else:
        Aqk, Akk = _gated(Q, K, gam, strict=False), _gated(K, K, gam, strict=True)
    G = gam.exp()
    Qh = Q * G * scale
    Kt = K * (gam[..., -1:, :] - gam).exp()
    A = Aqk * scale
    if not delta:
        return torch.zeros_like(K), Qh, Kt, A, V, G[..., -1, :]
    b = beta.float().reshape(B, N, CHUNK, H).permute(0, 3, 1, 2)[..., None]   # (B, H, N, C, 1)
    Akk = Akk * b
    Tm = Akk + torch.eye(CHUNK, device=q.device, dtype=Akk.dtype)
    # T = (I + M)^-1 once (64 right-hand sides), then one batched product for
    # both W and U: far cheaper than a triangular solve with dk + dv columns
    eye = torch.eye(CHUNK, device=q.device, dtype=Akk.dtype).expand_as(Tm)
    T = torch.linalg.solve_triangular(Tm, eye, upper=False, unitriangular=True)
    WU = T @ torch.cat([b * K * G, b * V], dim=-1)
    W, U = WU[..., :dk], WU[..., dk:]
    return W, Qh, Kt, A, U, G[..., -1, :]


class _KDARec(torch.autograd.Function):
    """The state recurrence on the GDR kernels (per-channel decay)."""

    @staticmethod
    def forward(ctx, W, Qh, Kt, A, U, gam, S0, H: int):
        B, Hh, N, C, dk = W.shape
        dv = U.shape[-1]
        f16 = lambda t: t.to(torch.bfloat16).reshape(B * Hh, *t.shape[2:]).contiguous()   # noqa: E731
        W16, Qh16, Kt16, A16, U16 = (f16(t) for t in (W, Qh, Kt, A, U))
        gf = gam.float().reshape(B * Hh, N, dk).contiguous()
        S0f = None if S0 is None else S0.float().reshape(B * Hh, dk, dv).contiguous()
        o, Vp, states, S_out = native().gdr_rec_fwd(W16, Qh16, Kt16, A16, U16, gf, S0f, True, H)
        ctx.save_for_backward(W16, Qh16, Kt16, A16, Vp, gf, states)
        ctx.shape = (B, Hh, N, C, dk, dv)
        ctx.has_S0 = S0 is not None
        return o, S_out.view(B, Hh, dk, dv)

    @staticmethod
    def backward(ctx, do, dS):
        W16, Qh16, Kt16, A16, Vp, gf, states = ctx.saved_tensors
        B, Hh, N, C, dk, dv = ctx.shape
        dO = do.to(torch.bfloat16).contiguous()
        dSf = None if dS is None else dS.float().reshape(B * Hh, dk, dv).contiguous()
        dW, dQh, dKt, dA, dU, dg, dS0 = native().gdr_rec_bwd(W16, Qh16, Kt16, A16, Vp, gf, states, dO, dSf,
                                                             ctx.has_S0)
        un = lambda t: t.float().view(B, Hh, N, *t.shape[2:])   # noqa: E731
        return (un(dW), un(dQh), un(dKt), un(dA), un(dU), dg.view(B, Hh, N, dk),
                dS0.view(B, Hh, dk, dv) if ctx.has_S0 else None, None)


def _kda_core_fwd(q, k, v, g, beta, S0, scale: float):
    """The fused KDA chunk forward: intra kernels + recurrence.  q, k, v bf16
    (B, L, H, .), g (B, L, H, dk) and beta (B, L, H) fp32.  Returns
    (o (B, L, H, dv) bf16, S (B * H, dk, dv) fp32, saved tensors)."""
    C = native()
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    W, Qh, Kt, A, U, gC = C.kda_intra_fwd(q, k, v, g, beta, scale)
    S0f = None if S0 is None else S0.float().reshape(B * H, dk, dv).contiguous()
    o, Vp, states, S_out = C.gdr_rec_fwd(W, Qh, Kt, A, U, gC, S0f, True, H)
    return o, S_out, (q, k, v, g, beta, W, Qh, Kt, A, Vp, gC, states)


def _kda_core_bwd(saved, do, dS, scale: float, need_dS0: bool):
    """(dq, dk, dv, dg, dbeta, dS0) of ``_kda_core_fwd``."""
    q, k, v, g, beta, W, Qh, Kt, A, Vp, gC, states = saved
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    C = native()
    dSf = None if dS is None else dS.float().reshape(B * H, dk, dv).contiguous()
    dW, dQh, dKt, dA, dU, dgC, dS0 = C.gdr_rec_bwd(W, Qh, Kt, A, Vp, gC, states,
                                                    do.to(torch.bfloat16).contiguous(), dSf, need_dS0)
    dq, dk_, dv_, dg, dbeta = C.kda_intra_bwd(q, k, v, g, beta, dW.to(torch.bfloat16), dQh.to(torch.bfloat16),
                                               dKt.to(torch.bfloat16), dA, dU.to(torch.bfloat16), dgC, scale)
    return dq, dk_, dv_, dg, dbeta, dS0


class _KDAFused(torch.autograd.Function):
    """The whole chunked KDA layer on our kernels: the intra-chunk stage
    (``kda_intra.cu``: per-channel cumulative decay, gated products, WY
    transform) and the state recurrence (``gdr.cu``), forward and backward,
    with no autograd graph in between.  q, k (B, L, H, dk), v (B, L, H, dv)
    bf16, g (B, L, H, dk) and beta (B, L, H) fp32, L a multiple of 64."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, S0, scale: float):
        B, L, H, dk = q.shape
        dv = v.shape[-1]
        o, S_out, saved = _kda_core_fwd(q, k, v, g, beta, S0, scale)
        ctx.save_for_backward(*saved)
        ctx.scale, ctx.has_S0, ctx.shape = scale, S0 is not None, (B, H, dk, dv)
        return o, S_out.view(B, H, dk, dv)

    @staticmethod
    def backward(ctx, do, dS):
        B, H, dk, dv = ctx.shape
        dq, dk_, dv_, dg, dbeta, dS0 = _kda_core_bwd(ctx.saved_tensors, do, dS, ctx.scale, ctx.has_S0)
        return dq, dk_, dv_, dg, dbeta, (dS0.view(B, H, dk, dv) if ctx.has_S0 else None), None


def _fused_ok(q, v, delta, w) -> bool:
    return (q.is_cuda and delta and w is None and q.shape[-1] == 128 and v.shape[-1] in (128, 256)
            and q.shape[1] % CHUNK == 0)


def kda_chunk(q, k, v, g, beta, S0, *, scale: float, chunk_size: int = 64, delta: bool = True, w=None):
    """Chunked delta rule with a per-channel gate g (B, L, H, dk) (log decay)
    on CUDA; ``delta=False`` is gated linear attention (beta unused), and a
    scalar gate (B, L, H) or no gate (None) is broadcast over the channels.
    ``w`` (B, L, H, dk) is an explicit write vector (the asymmetric write of
    the Kalman diagonal gain; beta unused).
    Returns (o (B, L, H, dv) bf16, S (B, H, dk, dv) fp32)."""
    assert chunk_size == CHUNK, "the sm_100a recurrence runs 64-token chunks"
    B, L, H, dk = q.shape
    if g is None:
        g = torch.zeros(B, L, H, dk, device=q.device, dtype=torch.float32)
    elif g.dim() == 3:
        g = g.float()[..., None].expand(B, L, H, dk)
    if beta is None:
        beta = torch.zeros(B, L, H, device=q.device, dtype=torch.float32)
    pad = (-L) % CHUNK
    if pad:
        # zero gate and zero write strength: padded tokens leave the state alone
        pz = lambda t: torch.nn.functional.pad(t, [0, 0] * (t.dim() - 2) + [0, pad])   # noqa: E731
        q, k, v, g, beta = pz(q), pz(k), pz(v), pz(g), pz(beta)
        w = None if w is None else pz(w)
    if _fused_ok(q, v, delta, w):
        bf = lambda t: t.to(torch.bfloat16).contiguous()   # noqa: E731
        o, S = _KDAFused.apply(bf(q), bf(k), bf(v), g.float().contiguous(), beta.float().contiguous(), S0, scale)
        return (o[:, :L] if pad else o), S
    parts = kda_intra(q, k, v, g, beta, scale, delta, w)
    o, S = _KDARec.apply(*parts, S0, H)
    return (o[:, :L] if pad else o), S


# ------------------------------------------------------------- fused layer --

def _packed_weight_kda(m):
    """bf16 rows [wq; wk; wv; wg; wa1; wb; 0-pad] of a per-channel-gate layer:
    every projection of the layer input is one GEMM (the gate's second,
    low-rank factor wa2 runs on its output)."""
    from .gdn import _PAD
    ws = [m.wq.weight, m.wk.weight, m.wv.weight, m.wg.weight, m.wa1.weight, m.wb.weight]
    n = sum(w.shape[0] for w in ws)
    pad = (-n) % 64
    key = ("kda_pad", pad, m.dim)
    zeros = _PAD.get(key)
    if zeros is None or zeros.device != ws[0].device:
        zeros = torch.zeros(pad, m.dim, device=ws[0].device, dtype=torch.float32)
        _PAD[key] = zeros
    return BF16.get_cat(ws + [zeros]), n


class _KDAMixer(torch.autograd.Function):
    """h (B, L, D) bf16 -> the gated normalised head concat (B, L, H dv) of a
    per-channel-gate (KDA) layer.  Column layout of the packed projection P:
    [q | k | v | gate | a1 (rank R) | b | pad]; f = a1 wa2^T is the gate's
    pre-activation."""

    @staticmethod
    def forward(ctx, h, Wp, wq, wk, wv, wg, wa1, wb, wa2, A_log, dt_bias, cq, ck, cv, gamma, meta):
        H, dk, dv, R, eps, scale = meta
        B, L, Dm = h.shape
        Hk, Hv = H * dk, H * dv
        h2 = as_bf16_2d(h)
        T = h2.shape[0]
        NP = Wp.shape[0]
        P = torch.empty(T, NP, device=h.device, dtype=torch.bfloat16)
        gemm(h2, False, Wp, False, P)
        P3 = P.view(B, L, NP)
        oa = 2 * Hk + 2 * Hv                                  # a1 | b column offset
        a1 = P[:, oa:oa + R]
        w2 = BF16.get(wa2)
        F = torch.empty(T, Hk, device=h.device, dtype=torch.bfloat16)
        gemm(a1, False, w2, False, F)                         # f = a1 wa2^T
        C = native()
        g, beta = C.kda_gates_fwd(F, P[:, oa + R:oa + R + H], A_log, dt_bias, H, dk)
        cq, ck, cv = cq.float().contiguous(), ck.float().contiguous(), cv.float().contiguous()
        q, rq = C.conv_silu_fwd(P3[:, :, :Hk], cq, dk, True)
        k, rk = C.conv_silu_fwd(P3[:, :, Hk:2 * Hk], ck, dk, True)
        v, _ = C.conv_silu_fwd(P3[:, :, 2 * Hk:2 * Hk + Hv], cv, dv, False)
        o, _S, ksaved = _kda_core_fwd(q.view(B, L, H, dk), k.view(B, L, H, dk), v.view(B, L, H, dv),
                                      g.view(B, L, H, dk), beta.view(B, L, H), None, scale)
        o = o.contiguous()
        y, rstd = C.rmsnorm_gated_fwd(o.view(T, H, dv), P[:, 2 * Hk + Hv:oa], gamma.float().contiguous(), eps, H)
        ctx.dims = (B, L, Dm, H, dk, dv, R, NP)
        ctx.scale = scale
        ctx.save_for_backward(h2, Wp, P, F, w2, rq, rk, o, rstd, A_log, dt_bias, cq, ck, cv, gamma, *ksaved)
        return y.view(B, L, Hv)

    @staticmethod
    def backward(ctx, dy):
        B, L, Dm, H, dk, dv, R, NP = ctx.dims
        Hk, Hv = H * dk, H * dv
        oa = 2 * Hk + 2 * Hv
        sv = ctx.saved_tensors
        h2, Wp, P, F, w2, rq, rk, o, rstd, A_log, dt_bias, cq, ck, cv, gamma = sv[:15]
        ksaved = sv[15:]
        T = h2.shape[0]
        C = native()
        dP = torch.empty(T, NP, device=h2.device, dtype=torch.bfloat16)
        if NP > oa + R + H:
            dP[:, oa + R + H:].zero_()
        do, dgamma = C.rmsnorm_gated_bwd(dy.reshape(T, Hv).to(torch.bfloat16), o.view(T, H, dv),
                                         P[:, 2 * Hk + Hv:oa], gamma.float().contiguous(), rstd,
                                         dP[:, 2 * Hk + Hv:oa], H)
        gq, gk, gv, gg, gb, _ = _kda_core_bwd(ksaved, do.view(B, L, H, dv), None, ctx.scale, False)
        dF = torch.empty(T, Hk, device=h2.device, dtype=torch.bfloat16)
        dA_log, ddt = C.kda_gates_bwd(gg.reshape(T, Hk), gb.reshape(T, H), F, P[:, oa + R:oa + R + H], A_log,
                                      dt_bias, dF, dP[:, oa + R:oa + R + H], H, dk)
        gemm(dF, False, w2, True, dP[:, oa:oa + R])                          # da1 = df wa2
        dwa2 = torch.zeros(Hk, R, device=h2.device, dtype=torch.float32)
        gemm(dF, True, P[:, oa:oa + R], True, dwa2, atomic=True)             # dwa2 = df^T a1
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
        dwq, dwk, dwv, dwg, dwa1, dwb = dWp[:oa + R + H].split([Hk, Hk, Hv, Hv, R, H], 0)
        return (dh.view(B, L, Dm), None, dwq, dwk, dwv, dwg, dwa1, dwb, dwa2, dA_log, ddt.view_as(dt_bias),
                dcq.view_as(cq), dck.view_as(ck), dcv.view_as(cv), dgamma, None)


def kda_mixer(m, x):
    """Fused forward of a per-channel-gate delta-rule layer (short conv,
    softplus gate) up to the input of ``wo``."""
    B, L, _ = x.shape
    meta = (m.head_count, m.key_head_dim, m.value_head_dim, m.gate_rank, m.o_norm.eps, m.scale)
    pad = (-L) % CHUNK
    if pad:
        x = torch.nn.functional.pad(x, (0, 0, 0, pad))
    Wp, _ = _packed_weight_kda(m)
    y = _KDAMixer.apply(x.to(torch.bfloat16), Wp, m.wq.weight, m.wk.weight, m.wv.weight, m.wg.weight,
                        m.wa1.weight, m.wb.weight, m.wa2.weight, m.A_log, m.dt_bias, m.conv_q.conv.weight,
                        m.conv_k.conv.weight, m.conv_v.conv.weight, m.o_norm.gamma, meta)
    return y[:, :L] if pad else y
