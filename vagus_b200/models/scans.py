"""The gated delta-rule scans as pure functions -- the oracles every kernel is
checked against.

Per head, with state S in R^{dk x dv}, decay a_t and write strength b_t:

    S_t = (I - b_t k_t k_t^T) Diag(a_t) S_{t-1} + b_t k_t v_t^T
    o_t = scale * S_t^T q_t

``g`` carries log a_t: (B, L, H) for a scalar gate (Gated DeltaNet), (B, L, H,
dk) for a per-channel gate (KDA), or None (a_t = 1, DeltaNet).  ``delta=False``
drops the erase term (gated linear attention).  An explicit write vector ``w``
replaces b_t k_t in the write slot (the asymmetric rule a diagonal Kalman gain
produces).

Shapes: q, k (B, L, H, dk); v (B, L, H, dv); beta (B, L, H); S0 (B, H, dk, dv)
or None.  Return ``(o, S)``: o (B, L, H, dv) in q's dtype, S fp32 (fp64 when q
is fp64, the tests' exactness regime).

The chunked forms below are written from the algebra in the docstrings, not
from any kernel: within a chunk with cumulative log decay gamma_i and
D_ij = exp(gamma_i - gamma_j) (i >= j), the delta-rule product collapses to
one unit-lower-triangular solve

    T = (I + strict(diag(b) K K^T o D))^{-1}
    W = T diag(b G) K,   U = T diag(b) V           (G_i = exp(gamma_i))
    V' = U - W S0                                  (the "new values")
    O  = diag(G) Q S0 + (Q K^T o D)_causal V'
    S_C = G_C S0 + (K o (G_C / G))^T V'

which is what the sm_100a chunk kernels compute tile by tile.

Parity: reference ``infra/components/linear_attention.py:128-425``
(chunk_scan_flops, recurrent_scan, residual_scan, chunk_scan, chunk_scan_vec)
and the fusion-flag parser ``:70-125``.
"""

from __future__ import annotations

import torch
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

__all__ = [
    "FUSIONS", "parse_fusions", "chunk_scan_flops", "recurrent_scan", "residual_scan",
    "chunk_scan", "chunk_scan_vec",
]

# Fusion flags accepted in recipes (``la_fused``).  The sm_100a path always
# runs all of them fused (conv+SiLU+L2 norm in one kernel, the gate activation
# and beta sigmoid inside the projection epilogue, RMSNorm*SiLU(gate) in one
# kernel), so the flags only matter for recipe round-trips.
FUSIONS = ("conv", "l2norm", "gate", "beta", "norm_gate")
_ALIASES = {"scan": ("l2norm", "gate", "beta"), "all": FUSIONS}


def parse_fusions(spec) -> frozenset:
    """True (all), False/None (none), or a subset: 'gate', 'conv,gate',
    'scan', ['conv', 'gate']."""
    if spec is True:
        return frozenset(FUSIONS)
    if not spec:
        return frozenset()
    names = [s.strip() for s in spec.split(",")] if isinstance(spec, str) else list(spec)
    out: set[str] = set()
    for n in names:
        if n:
            out.update(_ALIASES.get(n, (n,)))
    bad = out - set(FUSIONS)
    assert not bad, f"unknown fusion {sorted(bad)}; pick from {FUSIONS} or {sorted(_ALIASES)}"
    return frozenset(out)


def chunk_scan_flops(dk: int, dv: int, chunk: int, delta: bool) -> float:
    """Matmul FLOPs per token per head, forward + backward (x3), of the
    chunkwise algorithm: the recurrence (state write, delta read-back, query
    read-out, 2 dk dv each) plus the intra-chunk products over a C-token
    chunk (Q K^T and the masked read 2C(dk + dv); with the delta rule also the
    K K^T gram and the two WY products, 2C(3 dk + 2 dv) in total)."""
    state = (6 if delta else 4) * dk * dv
    intra = 2 * chunk * ((3 * dk + 2 * dv) if delta else (dk + dv))
    return 3.0 * (state + intra)


def _work_dtype(q: torch.Tensor) -> torch.dtype:
    return torch.float64 if q.dtype == torch.float64 else torch.float32


def _decay_state(S: torch.Tensor, gt: torch.Tensor | None, dt: torch.dtype) -> torch.Tensor:
    if gt is None:
        return S
    a = gt.to(dt).exp()
    return S * (a[..., None] if a.dim() == 3 else a[..., None, None])


def recurrent_scan(q, k, v, g, beta, S0, *, scale: float, delta: bool, w=None):
    """Token-by-token recurrence: the definition everything else must match."""
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    dt = _work_dtype(q)
    qf, kf, vf = q.to(dt) * scale, k.to(dt), v.to(dt)
    S = q.new_zeros(B, H, dk, dv, dtype=dt) if S0 is None else S0.to(dt)
    outs = []
    for t in range(L):
        S = _decay_state(S, None if g is None else g[:, t], dt)
        kt, vt = kf[:, t], vf[:, t]
        if delta:
            if w is None:
                assert beta is not None
                wt = kt * beta[:, t].to(dt)[..., None]
            else:
                wt = w[:, t].to(dt)
            resid = vt - torch.einsum("bhk,bhkv->bhv", kt, S)
            S = S + wt[..., :, None] * resid[..., None, :]
        else:
            S = S + kt[..., :, None] * vt[..., None, :]
        outs.append(torch.einsum("bhk,bhkv->bhv", qf[:, t], S))
    o = torch.stack(outs, 1) if L else q.new_zeros(B, 0, H, dv, dtype=dt)
    return o.to(q.dtype), S


def residual_scan(k, v, g, beta, S0, *, delta: bool, w=None):
    """(B, L, H) delta-rule surprise ratios |v_t - S_{t-1}^T k_t| / |v_t|, with
    S_{t-1} already decayed (1 everywhere without the delta rule)."""
    B, L, H, dk = k.shape
    dv = v.shape[-1]
    dt = _work_dtype(k)
    kf, vf = k.to(dt), v.to(dt)
    S = k.new_zeros(B, H, dk, dv, dtype=dt) if S0 is None else S0.to(dt)
    out = []
    for t in range(L):
        S = _decay_state(S, None if g is None else g[:, t], dt)
        kt, vt = kf[:, t], vf[:, t]
        if delta:
            r = vt - torch.einsum("bhk,bhkv->bhv", kt, S)
            out.append(r.norm(dim=-1) / vt.norm(dim=-1).clamp(min=1e-6))
            wt = kt * beta[:, t].to(dt)[..., None] if w is None else w[:, t].to(dt)
            S = S + wt[..., :, None] * r[..., None, :]
        else:
            out.append(torch.ones(B, H, device=k.device, dtype=dt))
            S = S + kt[..., :, None] * vt[..., None, :]
    if not L:
        return k.new_zeros(B, 0, H, dtype=torch.float32)
    return torch.stack(out, 1).float()


def _to_chunks(t: torch.Tensor, C: int) -> torch.Tensor:
    """(B, N*C, H, d) -> (B, H, N, C, d)."""
    B, T, H, d = t.shape
    return t.view(B, T // C, C, H, d).permute(0, 3, 1, 2, 4)


def _pad_time(t, pad):
    if t is None or not pad:
        return t
    tail = [0, 0] * (t.dim() - 2) + [0, pad]
    return F.pad(t, tail)


def chunk_scan(q, k, v, g, beta, S0, *, scale: float, delta: bool, chunk_size: int = 64):
    """Chunkwise scan for a scalar (or no) gate; a per-channel gate dispatches
    to ``chunk_scan_vec``.  O(L / C) sequential steps."""
    if g is not None and g.dim() == 4:
        return chunk_scan_vec(q, k, v, g, beta, S0, scale=scale, delta=delta, chunk_size=chunk_size)
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    C = chunk_size
    dt = _work_dtype(q)
    pad = (-L) % C
    # padded positions are inert: q = k = v = 0, log a = 0, b = 0
    qf, kf, vf = (_pad_time(t.to(dt), pad) for t in (q, k, v))
    qf = qf * scale
    N = (L + pad) // C
    Q, K, V = _to_chunks(qf, C), _to_chunks(kf, C), _to_chunks(vf, C)
    if g is None:
        gam = qf.new_zeros(B, H, N, C)
    else:
        gam = _pad_time(g.to(dt), pad).view(B, N, C, H).permute(0, 3, 1, 2).cumsum(-1)
    causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    # mask before exp: the upper triangle holds positive exponents
    D = (gam[..., :, None] - gam[..., None, :]).masked_fill(~causal, float("-inf")).exp()
    Gi = gam.exp()                                    # G_i
    Gend = (gam[..., -1:] - gam).exp()                # G_C / G_i
    Aqk = (Q @ K.transpose(-1, -2)) * D
    if delta:
        b = _pad_time(beta.to(dt), pad).view(B, N, C, H).permute(0, 3, 1, 2)
        Akk = (b[..., :, None] * (K @ K.transpose(-1, -2)) * D).tril(-1)
        eye = torch.eye(C, dtype=dt, device=q.device)
        Tm = eye + Akk
        Wm = torch.linalg.solve_triangular(Tm, (b * Gi)[..., None] * K, upper=False, unitriangular=True)
        Um = torch.linalg.solve_triangular(Tm, b[..., None] * V, upper=False, unitriangular=True)
    else:
        Wm, Um = None, V
    S = qf.new_zeros(B, H, dk, dv) if S0 is None else S0.to(dt)
    outs = []
    for n in range(N):
        Vn = Um[:, :, n] if Wm is None else Um[:, :, n] - Wm[:, :, n] @ S
        outs.append(Gi[:, :, n, :, None] * (Q[:, :, n] @ S) + Aqk[:, :, n] @ Vn)
        S = Gi[:, :, n, -1, None, None] * S + (K[:, :, n] * Gend[:, :, n, :, None]).transpose(-1, -2) @ Vn
    if not outs:
        return q.new_zeros(B, 0, H, dv), S
    o = torch.stack(outs, 2).permute(0, 2, 3, 1, 4).reshape(B, N * C, H, dv)[:, :L]
    return o.to(q.dtype), S


def _vec_chunk(qn, kn, vn, wn, bn, gn, S, strict, causal, eye):
    """One chunk of the per-channel-gate scan.

    gn: (B, H, C, dk) cumulative log decay.  With E_ijc = exp(gn_i[c] - gn_j[c])
    (i >= j) every inner product becomes a gated one,
    <x_i, y_j>_g = sum_c x_i[c] y_j[c] E_ijc, whose exponents are <= 0.  The
    pairwise form is kept because factorising E overflows fp32 for fast
    channels."""
    E = (gn[:, :, :, None, :] - gn[:, :, None, :, :]).masked_fill(
        ~causal[None, None, :, :, None], float("-inf")).exp()            # (B, H, C, C, dk)
    G = gn.exp()
    Gend = (gn[:, :, -1:, :] - gn).exp()

    def gdot(a, b):
        return torch.einsum("bhic,bhijc,bhjc->bhij", a, E, b)

    if wn is not None:
        # asymmetric write: S_i = S_{i-1} + w_i r_i^T, r_i = v_i - S_{i-1}^T k_i
        M = gdot(kn, wn) * strict
        Tm = eye + M
        R = torch.linalg.solve_triangular(Tm, vn - (kn * G) @ S, upper=False, unitriangular=True)
        out = (qn * G) @ S + (gdot(qn, wn) * causal) @ R
        Snew = G[:, :, -1, :, None] * S + (wn * Gend).transpose(-1, -2) @ R
        return out, Snew
    if bn is not None:
        M = (bn[..., None] * gdot(kn, kn)) * strict
        Tm = eye + M
        Wm = torch.linalg.solve_triangular(Tm, bn[..., None] * kn * G, upper=False, unitriangular=True)
        Um = torch.linalg.solve_triangular(Tm, bn[..., None] * vn, upper=False, unitriangular=True)
        Vn = Um - Wm @ S
        out = (qn * G) @ S + (gdot(qn, kn) * causal) @ Vn
        Snew = G[:, :, -1, :, None] * S + (kn * Gend).transpose(-1, -2) @ Vn
        return out, Snew
    out = (qn * G) @ S + (gdot(qn, kn) * causal) @ vn
    Snew = G[:, :, -1, :, None] * S + (kn * Gend).transpose(-1, -2) @ vn
    return out, Snew


def chunk_scan_vec(q, k, v, g, beta, S0, *, scale: float, delta: bool, chunk_size: int = 64, w=None):
    """Chunkwise scan for a per-channel gate g (B, L, H, dk) (KDA), with an
    optional explicit write vector ``w`` (k stays in the reading slot, w takes
    the writing slot).  Each chunk body is gradient-checkpointed when autograd
    is recording: its (B, H, C, C, dk) pairwise-decay tensor would otherwise
    be held once per chunk per layer."""
    B, L, H, dk = q.shape
    dv = v.shape[-1]
    C = chunk_size
    dt = _work_dtype(q)
    pad = (-L) % C
    qf = _pad_time(q.to(dt) * scale, pad)
    kf, vf, gf = (_pad_time(t.to(dt), pad) for t in (k, v, g))
    N = (L + pad) // C
    if w is not None:
        assert delta, "an explicit write vector needs the delta rule"
        w = _to_chunks(_pad_time(w.to(dt), pad), C)
    Q, K, V = _to_chunks(qf, C), _to_chunks(kf, C), _to_chunks(vf, C)
    gam = _to_chunks(gf, C).cumsum(3)
    causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    strict = causal.tril(-1)
    eye = torch.eye(C, dtype=dt, device=q.device)
    b = None
    if delta and w is None:
        assert beta is not None
        b = _pad_time(beta.to(dt), pad).view(B, N, C, H).permute(0, 3, 1, 2)
    S = qf.new_zeros(B, H, dk, dv) if S0 is None else S0.to(dt)
    ckpt = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (q, k, v, g, w, beta))
    outs = []
    for n in range(N):
        args = (Q[:, :, n], K[:, :, n], V[:, :, n], None if w is None else w[:, :, n],
                None if b is None else b[:, :, n], gam[:, :, n], S, strict, causal, eye)
        if ckpt:
            on, S = checkpoint(_vec_chunk, *args, use_reentrant=False)
        else:
            on, S = _vec_chunk(*args)
        outs.append(on)
    if not outs:
        return q.new_zeros(B, 0, H, dv), S
    o = torch.stack(outs, 2).permute(0, 2, 3, 1, 4).reshape(B, N * C, H, dv)[:, :L]
    return o.to(q.dtype), S
