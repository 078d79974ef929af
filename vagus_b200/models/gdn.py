"""The gated delta-rule token mixer (KDA, Gated DeltaNet, DeltaNet, GLA-like).

Layout per layer:

    q, k = L2norm(SiLU(conv(W x))) per head;  v = SiLU(conv(W x))
    a_t  = exp(-exp(A_log) softplus(f(x) + dt_bias))            [gate]
           f = W_a x (scalar gate) or W_a2 W_a1 x (vector gate, low rank)
           bounded form: lower_bound * sigmoid(exp(A_log) (f + dt_bias))
    b_t  = sigmoid(W_b x)                                        [delta]
    out  = W_o (RMSNorm_head(scan(q, k, v)) * SiLU(W_g x))

Mamba2-style init: A_log ~ log U(A_init_range) per head, dt_bias the inverse
activation of dt ~ logU(dt_init_range) (per channel for the vector gate, per
head for the scalar gate).  Projections N(0, init_std), wo shrunk by
1/sqrt(2 L).

Execution on CUDA (``impl`` 'auto'/'cuda'): the forward of a scalar-gate delta
layer runs as sm_100a kernels -- one projection GEMM for q/k/v/g, one fused
short-conv+SiLU+L2norm kernel, the gate/beta kernel, the chunked gated
delta-rule kernel and the fused RMSNorm*SiLU(gate) kernel -- see
``vagus_b200.ops.gdn``.  The other variants on CUDA -- per-channel gate (KDA),
no gate (DeltaNet), no delta rule (gated linear attention), and the Kalman
writes (a per-head gain, or an explicit write vector) -- run their
intra-chunk stage chunk-parallel (gated products on ``csrc/kda.cu``; in
torch for an explicit write vector) and
the state recurrence on the same kernels (``vagus_b200.ops.kda``).  CPU and
fp64 runs use the pure-torch chunk oracles of ``models.scans``.

Parity: reference ``infra/components/linear_attention.py:505-952``.
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F

from .. import ops
from ..utils import infer_device, infer_dtype
from .conv import ShortConv
from .mixer import Mixer
from .norm import RMSNorm
from .scans import chunk_scan, chunk_scan_vec, parse_fusions, recurrent_scan, residual_scan

GATES = ("none", "scalar", "vector")
IMPLS = ("auto", "cuda", "torch", "fla")   # 'fla' is read as 'cuda' (recipe compatibility)


def _hi(x: torch.Tensor) -> torch.Tensor:
    """At least fp32 (bf16 -> fp32; fp64 stays fp64)."""
    return x.to(torch.promote_types(x.dtype, torch.float32))


def _l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    h = _hi(x)
    return (h * torch.rsqrt(h.pow(2).sum(-1, keepdim=True) + eps)).to(x.dtype)


class GatedDeltaNet(nn.Module, Mixer):
    def __init__(self, dim: int, head_count: int, key_head_dim: int, value_head_dim: int,
                 short_conv_size: int | None = 4, gate: str | bool = "vector", delta: bool = True,
                 gate_rank: int = 64, chunk_size: int = 64, impl: str = "auto",
                 fused: bool | str | list = False, conv_impl: str = "conv1d",
                 disable_recompute: bool = False, gate_lower_bound: float | None = None, *,
                 init_std: float = 0.02, layer_count: int | None = None,
                 A_init_range: tuple[float, float] = (1.0, 16.0),
                 dt_init_range: tuple[float, float] = (1e-3, 1e-1), out_proj: bool = True):
        super().__init__()
        if isinstance(gate, bool):            # legacy spelling: True = scalar
            gate = "scalar" if gate else "none"
        assert gate in GATES, gate
        assert dim > 0 and head_count > 0 and key_head_dim > 0 and value_head_dim > 0
        assert impl in IMPLS, impl
        assert gate_lower_bound is None or gate == "vector", \
            "the bounded decay is a KDA (vector-gate) parameterisation"
        assert gate_lower_bound is None or -5 <= gate_lower_bound < 0, \
            f"gate_lower_bound must be in [-5, 0), got {gate_lower_bound}"
        self.dim = dim
        self.head_count = head_count
        self.key_head_dim = key_head_dim
        self.value_head_dim = value_head_dim
        self.short_conv_size = short_conv_size
        self.gate = gate
        self.delta = delta
        self.gate_rank = gate_rank
        self.chunk_size = chunk_size
        self.impl = "cuda" if impl == "fla" else impl
        self.fusions = parse_fusions(fused)
        self.disable_recompute = disable_recompute
        self.gate_lower_bound = gate_lower_bound
        self.scale = key_head_dim ** -0.5
        self.out_proj = out_proj
        self.out_width = head_count * value_head_dim

        H, dk, dv = head_count, key_head_dim, value_head_dim
        self.wq = nn.Linear(dim, H * dk, bias=False)
        self.wk = nn.Linear(dim, H * dk, bias=False)
        self.wv = nn.Linear(dim, H * dv, bias=False)
        self.wg = nn.Linear(dim, H * dv, bias=False)
        if out_proj:
            self.wo = nn.Linear(H * dv, dim, bias=False)
        self.o_norm = RMSNorm(dv)
        if short_conv_size is not None:
            self.conv_q = ShortConv(H * dk, short_conv_size, impl=conv_impl)
            self.conv_k = ShortConv(H * dk, short_conv_size, impl=conv_impl)
            self.conv_v = ShortConv(H * dv, short_conv_size, impl=conv_impl)
        if gate != "none":
            n_dt = H * dk if gate == "vector" else H
            if gate == "vector":
                self.wa1 = nn.Linear(dim, gate_rank, bias=False)
                self.wa2 = nn.Linear(gate_rank, H * dk, bias=False)
            else:
                self.wa = nn.Linear(dim, H, bias=False)
            A = torch.empty(H).uniform_(*A_init_range)
            self.A_log = nn.Parameter(A.log())
            lo, hi = math.log(dt_init_range[0]), math.log(dt_init_range[1])
            dt = torch.exp(torch.rand(n_dt) * (hi - lo) + lo).clamp(min=1e-4)
            if gate_lower_bound is None:
                bias = dt + torch.log(-torch.expm1(-dt))          # softplus^-1(dt)
            else:
                # the bounded gate at f = 0 must give the same decay rate A dt:
                # -lb sigmoid(A b) = A dt  =>  b = logit(A dt / -lb) / A
                a = A.repeat_interleave(dk)
                p = (a * dt / -gate_lower_bound).clamp(1e-6, 1 - 1e-6)
                bias = torch.logit(p) / a
            self.dt_bias = nn.Parameter(bias)
        if delta:
            self.wb = nn.Linear(dim, H, bias=False)

        for lin in (self.wq, self.wk, self.wv, self.wg):
            nn.init.normal_(lin.weight, std=init_std)
        for name in ("wa", "wa1", "wa2", "wb"):
            if hasattr(self, name):
                nn.init.normal_(getattr(self, name).weight, std=init_std)
        if out_proj:
            nn.init.normal_(self.wo.weight, std=init_std / math.sqrt(2 * layer_count) if layer_count else init_std)

        self.cache_len = 0
        self.register_buffer("state", torch.zeros(0, 0, 0, 0), persistent=False)
        if short_conv_size is not None:
            self.register_buffer("qp_cache", torch.zeros(0, short_conv_size, H * dk), persistent=False)
            self.register_buffer("kp_cache", torch.zeros(0, short_conv_size, H * dk), persistent=False)
            self.register_buffer("vp_cache", torch.zeros(0, short_conv_size, H * dv), persistent=False)

    # --- pieces ----------------------------------------------------------

    @property
    def gate_projections(self) -> list[nn.Parameter]:
        """The skinny gate / beta matrices (routed to AdamW by default)."""
        return [getattr(self, n).weight for n in ("wa", "wa1", "wa2", "wb") if hasattr(self, n)]

    def _gates(self, x):
        """(g, beta): log decay (fp32, or fp64 for fp64 models) and write
        strength, each None when the layer has no such term."""
        g = beta = None
        if self.gate == "scalar":
            g = -_hi(self.A_log).exp() * F.softplus(_hi(ops.linear(x, self.wa.weight)) + _hi(self.dt_bias))
        elif self.gate == "vector":
            B, L = x.shape[0], x.shape[1]
            f = _hi(ops.linear(ops.linear(x, self.wa1.weight), self.wa2.weight)) + _hi(self.dt_bias)
            f = f.view(B, L, self.head_count, self.key_head_dim)
            A = _hi(self.A_log).exp()[:, None]
            if self.gate_lower_bound is not None:
                g = self.gate_lower_bound * torch.sigmoid(A * f)
            else:
                g = -A * F.softplus(f)
        if self.delta and hasattr(self, "wb"):
            beta = torch.sigmoid(_hi(ops.linear(x, self.wb.weight)))
        return g, beta

    def _heads(self, qp, kp, vp, *, conv: bool = True):
        B, L = qp.shape[0], qp.shape[1]
        H, dk, dv = self.head_count, self.key_head_dim, self.value_head_dim
        if conv and self.short_conv_size is not None and self._use_kernels(qp):
            # conv + SiLU (+ L2 norm of q, k) on the conv kernels
            q = ops.conv_silu(qp, self.conv_q.conv.weight, dk, True).view(B, L, H, dk)
            k = ops.conv_silu(kp, self.conv_k.conv.weight, dk, True).view(B, L, H, dk)
            return q, k, ops.conv_silu(vp, self.conv_v.conv.weight, dv, False).view(B, L, H, dv)
        if conv and self.short_conv_size is not None:
            qp, kp, vp = self.conv_q(qp, "silu"), self.conv_k(kp, "silu"), self.conv_v(vp, "silu")
        else:
            qp, kp, vp = F.silu(qp), F.silu(kp), F.silu(vp)
        q = _l2norm(qp.view(B, L, H, dk))
        k = _l2norm(kp.view(B, L, H, dk))
        return q, k, vp.view(B, L, H, dv)

    def _write(self, x, k, g, beta):
        """(beta, w): the write of this block.  The family's own write is the
        symmetric b_t k_t (w None); KalmanDeltaNet overrides this."""
        return beta, None

    def _scan(self, q, k, v, g, beta, S0, *, w=None):
        if w is not None:
            assert self.delta and g is not None and g.dim() == 4, \
                "the asymmetric chunk form is implemented for the vector gate"
            if self._use_kernels(q):
                return ops.kda_chunk(q, k, v, g, None, S0, scale=self.scale, chunk_size=self.chunk_size, w=w)
            return chunk_scan_vec(q, k, v, g, None, S0, scale=self.scale, delta=True,
                                  chunk_size=self.chunk_size, w=w)
        if self._use_kernels(q) and self.gate == "scalar" and self.delta:
            return ops.gdr_chunk(q, k, v, g, beta, S0, scale=self.scale, chunk_size=self.chunk_size)
        if self._use_kernels(q):
            # per-channel gate, no gate (DeltaNet), or no delta rule (gated linear attention):
            # the chunk-parallel intra stage in torch + gated products and the recurrence on the kernels
            return ops.kda_chunk(q, k, v, g, beta, S0, scale=self.scale, chunk_size=self.chunk_size,
                                 delta=self.delta)
        return chunk_scan(q, k, v, g, beta, S0, scale=self.scale, delta=self.delta,
                          chunk_size=self.chunk_size)

    def _output(self, o, x):
        B, L = x.shape[0], x.shape[1]
        gate = ops.linear(x, self.wg.weight).view(B, L, self.head_count, self.value_head_dim)
        o = ops.rmsnorm_gated(o.to(gate.dtype), gate, self.o_norm.gamma, self.o_norm.eps).reshape(B, L, -1)
        return ops.linear(o, self.wo.weight) if self.out_proj else o

    def _use_kernels(self, t: torch.Tensor) -> bool:
        """The sm_100a scan kernels take dk in {128, 256}, dv a multiple of 64
        and 64-token chunks."""
        return (t.is_cuda and self.impl != "torch" and t.dtype in (torch.bfloat16, torch.float16)
                and self.key_head_dim in (128, 256) and self.value_head_dim % 64 == 0 and self.chunk_size == 64)

    def _fused_ok(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and self.impl != "torch" and self.gate == "scalar" and self.delta
                and self.short_conv_size is not None and type(self)._write is GatedDeltaNet._write
                and self.key_head_dim in (128, 256) and self.value_head_dim % 64 == 0 and self.chunk_size == 64
                and self.dim % 64 == 0 and x.shape[0] * x.shape[1] >= 128)

    def _fused_kda_ok(self, x: torch.Tensor) -> bool:
        """The fused per-channel-gate layer (``ops.kda_mixer``): softplus gate,
        delta rule, short conv, key head dim 128, value head dim 128 / 256."""
        return (x.is_cuda and self.impl != "torch" and self.gate == "vector" and self.delta
                and self.gate_lower_bound is None and self.short_conv_size is not None
                and type(self)._write is GatedDeltaNet._write and self.key_head_dim == 128
                and self.value_head_dim in (128, 256) and self.chunk_size == 64 and self.dim % 64 == 0
                and self.gate_rank % 8 == 0 and self.gate_rank >= 64 and x.shape[0] * x.shape[1] >= 128)

    def _mixer(self, x):
        """The gated, normalised head concat on a fused path, or None."""
        if self._fused_ok(x):
            return ops.gdn_mixer(self, x)
        if self._fused_kda_ok(x):
            return ops.kda_mixer(self, x)
        return None

    # --- training / stateless ---------------------------------------------

    def forward(self, x, is_causal: bool = True):
        assert is_causal, "linear attention is causal by construction"
        o = self._mixer(x)
        if o is not None:
            return ops.linear(o, self.wo.weight) if self.out_proj else o
        qp, kp, vp = ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight), ops.linear(x, self.wv.weight)
        q, k, v = self._heads(qp, kp, vp)
        g, beta = self._gates(x)
        beta, w = self._write(x, k, g, beta)
        o, _ = self._scan(q, k, v, g, beta, None, w=w)
        return self._output(o, x)

    def forward_pre_out(self, x, is_causal: bool = True):
        """The gated, normalised head concat (the input of ``wo``).  Lets a
        block fuse ``wo`` with its residual add."""
        o = self._mixer(x)
        if o is not None:
            return o
        qp, kp, vp = ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight), ops.linear(x, self.wv.weight)
        q, k, v = self._heads(qp, kp, vp)
        g, beta = self._gates(x)
        beta, w = self._write(x, k, g, beta)
        o, _ = self._scan(q, k, v, g, beta, None, w=w)
        B, L = x.shape[0], x.shape[1]
        gate = ops.linear(x, self.wg.weight).view(B, L, self.head_count, self.value_head_dim)
        return ops.rmsnorm_gated(o.to(gate.dtype), gate, self.o_norm.gamma, self.o_norm.eps).reshape(B, L, -1)

    @torch.no_grad()
    def residuals(self, x) -> torch.Tensor:
        """(B, L, H) delta-rule surprise ratios along a fresh stream (torch path)."""
        q, k, v = self._heads(ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight),
                              ops.linear(x, self.wv.weight))
        g, beta = self._gates(x)
        beta, w = self._write(x, k, g, beta)
        return residual_scan(k, v, g, beta, None, delta=self.delta, w=w)

    @torch.no_grad()
    def gate_stats(self, x) -> dict:
        """Health probe on a small input: mean decay per head (per channel for
        a vector gate), memory length 1/(1-a), mean write strength, state RMS."""
        q, k, v = self._heads(ops.linear(x, self.wq.weight), ops.linear(x, self.wk.weight),
                              ops.linear(x, self.wv.weight))
        g, beta = self._gates(x)
        beta, w = self._write(x, k, g, beta)
        qf, kf, vf = q.float(), k.float(), v.float()
        if w is None:
            _, S = chunk_scan(qf, kf, vf, g, beta, None, scale=self.scale, delta=self.delta,
                              chunk_size=self.chunk_size)
        else:
            _, S = recurrent_scan(qf, kf, vf, g, beta, None, scale=self.scale, delta=self.delta, w=w)
        out = {"state_rms": S.pow(2).mean().sqrt()}
        if g is not None:
            a = g.exp().mean(dim=(0, 1)).flatten()
            out["alpha"] = a
            out["mem_len"] = 1.0 / (1.0 - a).clamp(min=1e-6)
        if w is not None:
            out["beta"] = w.norm(dim=-1).mean(dim=(0, 1))
        elif beta is not None:
            out["beta"] = beta.mean(dim=(0, 1))
        return out

    # --- streaming ---------------------------------------------------------

    def reset_cache(self, batch_size: int, max_cache_len: int | None = None):
        """``max_cache_len`` is accepted for interface parity: the state is fixed-size."""
        device, dtype = infer_device(self), infer_dtype(self)
        H, dk, dv = self.head_count, self.key_head_dim, self.value_head_dim
        self.cache_len = 0
        sdt = torch.float64 if dtype == torch.float64 else torch.float32
        self.state = torch.zeros(batch_size, H, dk, dv, device=device, dtype=sdt)
        if self.short_conv_size is not None:
            K = self.short_conv_size
            self.qp_cache = torch.zeros(batch_size, K, H * dk, device=device, dtype=dtype)
            self.kp_cache = torch.zeros(batch_size, K, H * dk, device=device, dtype=dtype)
            self.vp_cache = torch.zeros(batch_size, K, H * dv, device=device, dtype=dtype)

    def load_cache(self, cache: dict, max_cache_len: int | None = None):
        self.reset_cache(cache["state"].shape[0], max_cache_len)
        self.cache_len = int(cache["cache_len"])
        self.state.copy_(cache["state"])
        if self.short_conv_size is not None:
            self.qp_cache.copy_(cache["qp_cache"])
            self.kp_cache.copy_(cache["kp_cache"])
            self.vp_cache.copy_(cache["vp_cache"])

    def export_cache(self) -> dict:
        cache = {"state": self.state.clone(), "cache_len": self.cache_len}
        if self.short_conv_size is not None:
            cache.update(qp_cache=self.qp_cache.clone(), kp_cache=self.kp_cache.clone(),
                         vp_cache=self.vp_cache.clone())
        return cache

    @torch.no_grad()
    def decode_step(self, x):
        """Consume the next block (B, L, dim).  L == 1 runs one recurrent step
        (the single-token decode kernel on CUDA); longer blocks run the chunk
        scan from the current state."""
        B, L = x.shape[0], x.shape[1]
        assert self.state.shape[0] > 0, "No state allocated. Call reset_cache or load_cache first."
        assert B == self.state.shape[0], "Batch size does not match the state. Reset or load cache first."
        if L == 0:
            return x
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
        q, k, v = self._heads(qp, kp, vp, conv=False)
        g, beta = self._gates(x)
        beta, w = self._write(x, k, g, beta)
        if L == 1 and w is None and self._use_kernels(q) and self.delta and self.gate == "scalar":
            o, S = ops.gdr_decode(q, k, v, g, beta, self.state, scale=self.scale)
        elif L == 1:
            o, S = recurrent_scan(q, k, v, g, beta, self.state, scale=self.scale, delta=self.delta, w=w)
        else:
            o, S = self._scan(q, k, v, g, beta, self.state, w=w)
        self.state.copy_(S)
        self.cache_len += L
        return self._output(o, x)
