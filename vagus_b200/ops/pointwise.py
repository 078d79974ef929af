"""Normalisation, activation and embedding ops: a CPU oracle written in plain
PyTorch and, on CUDA, one fused sm_100a kernel per direction."""

from __future__ import annotations

import torch
from torch.nn import functional as F

from ._core import native


# ------------------------------------------------------------------ RMSNorm --

def _rmsnorm_ref(x, gamma, eps):
    dt = x.dtype
    h = x.to(torch.promote_types(dt, torch.float32))
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return h.to(dt) * gamma


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, eps, out_f32):
        xc = x.contiguous()
        y, rstd = native().rmsnorm_fwd(xc, gamma.float().contiguous(), eps, out_f32)
        ctx.save_for_backward(xc, gamma, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, rstd = ctx.saved_tensors
        dx, dg = native().rmsnorm_bwd(dy.contiguous(), x, gamma.float().contiguous(), rstd, None,
                                      x.dtype == torch.float32, False)
        return dx, dg.to(gamma.dtype), None, None


def rmsnorm(x, gamma, eps: float = 1e-6, out_dtype=None):
    """``(x * rsqrt(mean(x^2) + eps)) * gamma``, statistics in >= fp32.
    ``out_dtype`` (CUDA) selects the output precision (default: x's)."""
    if not x.is_cuda or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[-1] > 16384:
        y = _rmsnorm_ref(x, gamma, eps)
        return y if out_dtype is None else y.to(out_dtype)
    out_dtype = out_dtype or x.dtype
    if out_dtype not in (torch.float32, torch.bfloat16):
        return _rmsnorm_ref(x, gamma, eps).to(out_dtype)
    return _RMSNorm.apply(x, gamma, float(eps), out_dtype == torch.float32)


class _RMSNormPass(torch.autograd.Function):
    """``(rmsnorm(x) in bf16, x)`` as one autograd node.  A pre-norm block
    reads the residual stream twice (the norm and the residual add); with
    both uses behind this node the backward receives both gradients at once
    and the norm kernel adds them, instead of a separate add over the fp32
    stream.  It also writes a bf16 copy of the summed gradient, attached to
    the returned tensor as ``_vagus_bf16``, for the GEMM backward that
    consumes it next (``ops.linear_residual``)."""

    @staticmethod
    def forward(ctx, x, gamma, eps):
        xc = x.contiguous()
        y, rstd = native().rmsnorm_fwd(xc, gamma.float().contiguous(), eps, False)
        ctx.save_for_backward(xc, gamma, rstd)
        return y, x.view_as(x)

    @staticmethod
    def backward(ctx, dy, dpass):
        x, gamma, rstd = ctx.saved_tensors
        dres = None if dpass is None else dpass.float().contiguous()
        out = native().rmsnorm_bwd(dy.contiguous(), x, gamma.float().contiguous(), rstd, dres, True, True)
        dx, dg = out[0], out[1]
        if len(out) > 2:
            dx._vagus_bf16 = (out[2], dx._version)    # stale once dx is modified in place
        return dx, dg.to(gamma.dtype), None


def rmsnorm_pass(x, gamma, eps: float = 1e-6):
    """Returns ``(rmsnorm(x) as bf16, x)``; see ``_RMSNormPass``.  Falls back
    to the plain composition where the fused backward does not apply."""
    if (x.is_cuda and x.dtype == torch.float32 and x.shape[-1] in (512, 768, 1024, 1536, 2048)
            and torch.is_grad_enabled() and x.requires_grad):
        return _RMSNormPass.apply(x, gamma, float(eps))
    return rmsnorm(x, gamma, eps, out_dtype=torch.bfloat16 if x.is_cuda else None), x


# ------------------------------------------------------ gated RMSNorm (GDN) --

class _RMSNormGated(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, g, gamma, eps):
        oc, gc = o.contiguous(), g.contiguous()
        D = o.shape[-1]
        H = oc.shape[-2] if oc.dim() >= 2 else 1
        y, rstd = native().rmsnorm_gated_fwd(oc, gc.view(-1, H * D), gamma.float().contiguous(), eps, H)
        ctx.save_for_backward(oc, gc, gamma, rstd)
        ctx.H = H
        return y

    @staticmethod
    def backward(ctx, dy):
        o, g, gamma, rstd = ctx.saved_tensors
        H, D = ctx.H, o.shape[-1]
        dg = torch.empty_like(g)
        do, dgam = native().rmsnorm_gated_bwd(dy, o, g.view(-1, H * D), gamma.float().contiguous(), rstd,
                                              dg.view(-1, H * D), H)
        return do, dg, dgam.to(gamma.dtype), None


def rmsnorm_gated(o, g, gamma, eps: float = 1e-6):
    """``RMSNorm(o) * gamma * silu(g)`` over the last dim (per head)."""
    if o.is_cuda and o.dtype == torch.bfloat16 and g.dtype == torch.bfloat16:
        return _RMSNormGated.apply(o, g, gamma, float(eps))
    return _rmsnorm_ref(o, gamma, eps) * F.silu(g)


# ------------------------------------------------------------------- SwiGLU --

class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u):
        uc = u.contiguous()
        ctx.save_for_backward(uc)
        return native().swiglu_fwd(uc)

    @staticmethod
    def backward(ctx, ds):
        (u,) = ctx.saved_tensors
        return native().swiglu_bwd(ds, u)


def swiglu(u):
    """``silu(u1) * u2`` with ``[u1 | u2] = u`` split on the last dim."""
    if u.is_cuda and u.dtype == torch.bfloat16 and (u.shape[-1] // 2) % 2 == 0:
        return _SwiGLU.apply(u)
    a, b = torch.chunk(u, 2, dim=-1)
    return F.silu(a) * b


# ------------------------------------------------------------ sigmoid gate --

class _SigmoidGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g):
        xc, gc = x.contiguous(), g.contiguous()
        ctx.save_for_backward(xc, gc)
        return native().sigmoid_gate_fwd(xc, gc)

    @staticmethod
    def backward(ctx, dy):
        x, g = ctx.saved_tensors
        dx, dg = native().sigmoid_gate_bwd(dy, x, g)
        return dx, dg


def sigmoid_gate(x, g):
    if x.is_cuda and x.dtype == torch.bfloat16 and g.dtype == torch.bfloat16 and x.shape == g.shape:
        return _SigmoidGate.apply(x, g)
    return x * torch.sigmoid(g)


# ---------------------------------------------------------------- embedding --

class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, w):
        tc = tok.contiguous()
        ctx.save_for_backward(tc)
        ctx.wshape = w.shape
        return native().embedding_fwd(w.contiguous(), tc, True)

    @staticmethod
    def backward(ctx, dy):
        (tok,) = ctx.saved_tensors
        dW = torch.zeros(ctx.wshape, device=dy.device, dtype=torch.float32)
        native().embedding_bwd(dy, tok, dW)
        return None, dW


def embedding(tokens, w):
    if tokens.is_cuda and w.dtype == torch.float32:
        return _Embedding.apply(tokens, w)
    return F.embedding(tokens, w)


# ----------------------------------------------------- qk norm + RoPE --

def _qk_ref(x, gamma, tables, eps):
    if gamma is not None:
        x = _rmsnorm_ref(x, gamma, eps)
    if tables is not None:
        cos, sin = tables                      # (L, D/2)
        cos = cos[:, None, :].to(x.dtype) if cos.dtype != x.dtype else cos[:, None, :]
        sin = sin[:, None, :].to(x.dtype) if sin.dtype != x.dtype else sin[:, None, :]
        p = x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2)
        x0, x1 = p[..., 0], p[..., 1]
        x = torch.stack((x0 * cos - x1 * sin, x0 * sin + x1 * cos), -1).reshape(x.shape)
    return x


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, cos, sin, eps):
        xc = x.contiguous()
        g = None if gamma is None else gamma.float().contiguous()
        y, rstd = native().qk_norm_rope_fwd(xc, g, cos, sin, eps)
        ctx.save_for_backward(xc, gamma, cos, sin, rstd)
        ctx.has_gamma = gamma is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, cos, sin, rstd = ctx.saved_tensors
        g = gamma.float().contiguous() if ctx.has_gamma else None
        dx, dg = native().qk_norm_rope_bwd(dy, x, g, cos, sin, rstd)
        return dx, (dg.to(gamma.dtype) if ctx.has_gamma else None), None, None, None


def qk_norm_rope(x, gamma, tables, eps: float = 1e-6):
    """x: (B, L, H, D).  Optional per-head RMSNorm (gamma) then optional
    interleaved-pair RoPE with ``tables = (cos, sin)`` of shape (L, D/2).
    Returns bf16 on the CUDA path (the attention kernels' input)."""
    if gamma is None and tables is None:
        return x
    if x.is_cuda and x.dtype == torch.bfloat16:
        cos = sin = None
        if tables is not None:
            cos, sin = (t.float().contiguous() for t in tables)
        return _QKNormRope.apply(x, gamma, cos, sin, float(eps))
    return _qk_ref(x, gamma, tables, eps)
