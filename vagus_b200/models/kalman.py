"""Kalman delta networks: the delta rule's write strength replaced by a Kalman
gain computed from an uncertainty summary with its own cheap recurrence.

Isotropic (one precision scalar c per head):

    a_t    = mean_i alpha_ti^2                 (trace-projected decay)
    bhat_t = a_t / c_{t-1} + omega_t
    beta_t = bhat_t / (r_t + bhat_t |k_t|^2)
    c_t    = 1 / bhat_t + s |k_t|^2 / (dk r_t)

beta stays one scalar per head, so the memory scan is the plain delta rule.

Diagonal (one covariance per key channel):

    phat_t  = alpha_t^2 p_{t-1} + omega_t
    kappa_t = phat_t k_t / (r_t + sum_i phat_ti k_ti^2)
    p_t     = phat_t / (1 + s k_t^2 / r_t phat_t)

kappa is a vector not parallel to k: the asymmetric write, run by the chunked
vector-gate scan with an explicit ``w``.

Both uncertainty recurrences are Mobius maps x -> (A x + B) / (C x + D) with
non-negative coefficients (``mobius_scan``).  On CUDA fp32 they run on the
segmented scan kernel (``ops.mobius_scan``: segment maps composed as 2x2
products, then an exact replay of the recurrence); elsewhere as a torch
prefix product of the 2x2 matrices at log depth, renormalised after every
doubling step (a scalar multiple of the matrix is the same map) and blocked
so autograd never holds more than one block of the doubling tensors.

Parity: reference ``infra/components/kalman_delta.py:1-300``.
"""

from __future__ import annotations

import math
from functools import partial

import torch
import torch.nn.functional as F
from torch import nn

from .gdn import GatedDeltaNet, _hi

KALMAN = ("iso", "diag")
OMEGA_MIN = 0.05
R_MIN = 0.05
PRECISION_FLOOR = 0.1
PRECISION_INIT = 1.0


def _mobius_apply(M, x0):
    return (M[..., 0, 0] * x0 + M[..., 0, 1]) / (M[..., 1, 0] * x0 + M[..., 1, 1])


@torch._dynamo.disable
def mobius_scan(A, B, C, D, x0, *, impl: str = "parallel", block: int | None = 256):
    """x_t = (A_t x_{t-1} + B_t) / (C_t x_{t-1} + D_t) along dim 1.

    A..D: (B, L, *rest) non-negative; x0: (B, *rest); returns (B, L, *rest).
    'recurrent' is the definition (test oracle); 'parallel' is the log-depth
    prefix product (Hillis-Steele doubling on the 2x2 matrices), which on
    CUDA fp32 inputs runs as the segmented scan kernel (``ops.mobius_scan``);
    'torch' forces the doubling in torch."""
    L = A.shape[1]
    if impl == "parallel" and A.is_cuda and A.dtype == torch.float32 and L > 0:
        from .. import ops
        return ops.mobius_scan(A, B, C, D, x0)
    if impl == "torch":
        impl = "parallel"
    if impl == "recurrent":
        x, out = x0, []
        for t in range(L):
            x = (A[:, t] * x + B[:, t]) / (C[:, t] * x + D[:, t])
            out.append(x)
        return torch.stack(out, 1) if out else x0.new_zeros(x0.shape[0], 0, *x0.shape[1:])
    assert impl == "parallel", impl
    if block is not None and L > block:
        pieces, x = [], x0
        for lo in range(0, L, block):
            hi = min(lo + block, L)
            seg = mobius_scan(A[:, lo:hi], B[:, lo:hi], C[:, lo:hi], D[:, lo:hi], x, impl="torch", block=None)
            pieces.append(seg)
            x = seg[:, -1]
        return torch.cat(pieces, 1)
    M = torch.stack((torch.stack((A, B), -1), torch.stack((C, D), -1)), -2)   # (B, L, *rest, 2, 2)
    step = 1
    while step < L:
        # element t composes with the prefix ending at t - step
        M = torch.cat((M[:, :step], M[:, step:] @ M[:, :-step]), 1)
        M = M / M.abs().amax(dim=(-2, -1), keepdim=True).clamp(min=1e-30)
        step *= 2
    return _mobius_apply(M, x0[:, None])


def kalman_gain_iso(k, alpha, omega, r, c0, *, info_scale: float, impl: str = "parallel"):
    """k, alpha (decay, not log): (B, L, H, dk); omega, r: (B, L, H); c0: (B, H).
    Returns (beta (B, L, H), c_final (B, H))."""
    dk = k.shape[-1]
    a = alpha.square().mean(-1)
    kn2 = k.square().sum(-1)
    m = (info_scale / dk) * kn2 / r
    # c_t = (1 + m w) c_{t-1} + m a) / (w c_{t-1} + a) in Mobius form
    c = mobius_scan(1.0 + m * omega, m * a, omega, a, c0, impl=impl)
    c_prev = torch.cat((c0[:, None], c[:, :-1]), 1)
    bhat = a / c_prev + omega
    return bhat / (r + bhat * kn2), c[:, -1]


def kalman_gain_diag(k, alpha, omega, r, p0, *, info_scale: float, impl: str = "parallel"):
    """omega: (B, L, H, dk); r: (B, L, H); p0: (B, H, dk).
    Returns (kappa (B, L, H, dk), p_final (B, H, dk))."""
    a2 = alpha.square()
    wgt = info_scale * k.square() / r[..., None]
    p = mobius_scan(a2, omega, wgt * a2, 1.0 + wgt * omega, p0, impl=impl)
    p_prev = torch.cat((p0[:, None], p[:, :-1]), 1)
    phat = a2 * p_prev + omega
    kappa = phat * k / (r[..., None] + (phat * k.square()).sum(-1, keepdim=True))
    return kappa, p[:, -1]


class KalmanDeltaNet(GatedDeltaNet):
    """KDA with a Kalman gain in beta's place; the uncertainty state rides in
    the cache next to the memory (``gain_state``)."""

    def __init__(self, *args, kalman: str = "iso", omega_min: float = OMEGA_MIN, r_min: float = R_MIN,
                 info_scale: float | None = None, gain_impl: str = "parallel", **kw):
        assert kalman in KALMAN, f"kalman must be one of {KALMAN}, got {kalman!r}"
        kw.setdefault("gate", "vector")
        assert kw["gate"] == "vector", "KDN needs KDA's per-channel decay"
        assert kw.get("delta", True), "KDN is a delta-rule write"
        kw["delta"] = True
        super().__init__(*args, **kw)
        self.kalman = kalman
        self.omega_min = omega_min
        self.r_min = r_min
        self.gain_impl = gain_impl
        H, dk = self.head_count, self.key_head_dim
        self.info_scale = float(dk if info_scale is None else info_scale)
        del self.wb
        self.wr = nn.Linear(self.dim, H, bias=True)
        if kalman == "iso":
            self.womega = nn.Linear(self.dim, H, bias=True)
            nn.init.normal_(self.womega.weight, std=0.02)
        else:
            self.womega1 = nn.Linear(self.dim, self.gate_rank, bias=False)
            self.womega2 = nn.Linear(self.gate_rank, H * dk, bias=True)
            nn.init.normal_(self.womega1.weight, std=0.02)
            nn.init.zeros_(self.womega2.weight)
            nn.init.zeros_(self.womega2.bias)
        nn.init.normal_(self.wr.weight, std=0.02)
        self.c0_param = nn.Parameter(torch.full((H,), math.log(math.expm1(PRECISION_INIT - PRECISION_FLOOR))))
        self._entry_gain = None
        self.register_buffer("gain_state", torch.zeros(0, 0), persistent=False)

    @property
    def gate_projections(self) -> list[nn.Parameter]:
        names = ("wa", "wa1", "wa2", "wr", "womega", "womega1", "womega2")
        return [getattr(self, n).weight for n in names if hasattr(self, n)]

    def _entry_precision(self, B: int, device, dtype) -> torch.Tensor:
        c0 = (PRECISION_FLOOR + F.softplus(self.c0_param.float())).to(device=device, dtype=dtype)
        c0 = c0[None].expand(B, -1)
        if self.kalman == "iso":
            return c0
        return c0[..., None].expand(-1, -1, self.key_head_dim).reciprocal()

    def _gates(self, x):
        g, _ = super()._gates(x)
        return g, None

    def _noise(self, x, B: int, L: int):
        r = self.r_min + F.softplus(_hi(self.wr(x)))
        if self.kalman == "iso":
            omega = self.omega_min + F.softplus(_hi(self.womega(x)))
        else:
            raw = self.womega2(self.womega1(x)).view(B, L, self.head_count, self.key_head_dim)
            omega = self.omega_min + F.softplus(_hi(raw))
        return omega, r

    def _write(self, x, k, g, beta):
        assert g is not None, "KDN needs the decay"
        B, L = x.shape[0], x.shape[1]
        alpha = _hi(g).exp()
        omega, r = self._noise(x, B, L)
        kf = _hi(k)
        entry = self._entry_gain
        if entry is None:
            entry = self._entry_precision(B, x.device, alpha.dtype)
        fn = kalman_gain_iso if self.kalman == "iso" else kalman_gain_diag
        run = partial(fn, info_scale=self.info_scale, impl=self.gain_impl)
        if torch.is_grad_enabled() and alpha.requires_grad:
            gain, final = torch.utils.checkpoint.checkpoint(run, kf, alpha, omega, r, entry, use_reentrant=False)
        else:
            gain, final = run(kf, alpha, omega, r, entry)
        beta, w = (gain, None) if self.kalman == "iso" else (None, gain)
        if self._entry_gain is not None:
            self.gain_state.copy_(final)
        return beta, w

    def reset_cache(self, batch_size: int, max_cache_len: int | None = None):
        super().reset_cache(batch_size, max_cache_len)
        dev = self.state.device
        shape = (batch_size, self.head_count) + ((self.key_head_dim,) if self.kalman == "diag" else ())
        self.gain_state = torch.zeros(*shape, device=dev, dtype=torch.float32)
        self.gain_state.copy_(self._entry_precision(batch_size, dev, torch.float32))

    def load_cache(self, cache: dict, max_cache_len: int | None = None):
        super().load_cache(cache, max_cache_len)
        self.gain_state.copy_(cache["gain_state"])

    def export_cache(self) -> dict:
        return {**super().export_cache(), "gain_state": self.gain_state.clone()}

    @torch.no_grad()
    def decode_step(self, x):
        if x.shape[1] == 0:
            return x
        self._entry_gain = self.gain_state.clone()
        try:
            return super().decode_step(x)
        finally:
            self._entry_gain = None
