# The gated delta-rule oracles (CPU, fp64): chunk forms == token recurrence,
# gradients, reductions between gate kinds, and the module's streaming path.
import pytest
import torch
import torch.nn.functional as F

from vagus_b200.models.conv import ShortConv
from vagus_b200.models.gdn import GatedDeltaNet
from vagus_b200.models.scans import (chunk_scan, chunk_scan_flops, chunk_scan_vec, parse_fusions, recurrent_scan,
                                     residual_scan)


def inputs(B=2, L=37, H=2, dk=8, dv=6, gate="scalar", seed=0, dtype=torch.float64):
    g0 = torch.Generator().manual_seed(seed)
    q = torch.randn(B, L, H, dk, generator=g0, dtype=dtype)
    k = F.normalize(torch.randn(B, L, H, dk, generator=g0, dtype=dtype), dim=-1)
    v = torch.randn(B, L, H, dv, generator=g0, dtype=dtype)
    shape = (B, L, H) if gate == "scalar" else (B, L, H, dk)
    g = None if gate == "none" else F.logsigmoid(torch.randn(*shape, generator=g0, dtype=dtype) + 2)
    beta = torch.sigmoid(torch.randn(B, L, H, generator=g0, dtype=dtype))
    S0 = torch.randn(B, H, dk, dv, generator=g0, dtype=dtype) * 0.1
    return q, k, v, g, beta, S0


@pytest.mark.parametrize("gate", ["none", "scalar", "vector"])
@pytest.mark.parametrize("delta", [True, False])
@pytest.mark.parametrize("C", [8, 64])
def test_chunk_matches_recurrent(gate, delta, C):
    q, k, v, g, beta, S0 = inputs(gate=gate)
    o_r, S_r = recurrent_scan(q, k, v, g, beta, S0, scale=0.3, delta=delta)
    o_c, S_c = chunk_scan(q, k, v, g, beta, S0, scale=0.3, delta=delta, chunk_size=C)
    assert torch.allclose(o_c, o_r, atol=1e-11) and torch.allclose(S_c, S_r, atol=1e-11)


@pytest.mark.parametrize("gate", ["scalar", "vector"])
def test_chunk_gradients_match_recurrent(gate):
    ins = inputs(L=19, gate=gate)
    a = [t.clone().requires_grad_(True) for t in ins]
    b = [t.clone().requires_grad_(True) for t in ins]
    o1, S1 = recurrent_scan(*a[:5], a[5], scale=0.5, delta=True)
    o2, S2 = chunk_scan(*b[:5], b[5], scale=0.5, delta=True, chunk_size=8)
    w1, w2 = torch.randn_like(o1), torch.randn_like(S1)
    ((o1 * w1).sum() + (S1 * w2).sum()).backward()
    ((o2 * w1).sum() + (S2 * w2).sum()).backward()
    for x, y in zip(a, b):
        assert torch.allclose(x.grad, y.grad, atol=1e-10)


def test_vector_gate_reduces_to_scalar():
    q, k, v, g, beta, S0 = inputs(gate="scalar")
    gv = g[..., None].expand(*g.shape, k.shape[-1]).contiguous()
    o1, S1 = chunk_scan(q, k, v, g, beta, S0, scale=1.0, delta=True, chunk_size=8)
    o2, S2 = chunk_scan_vec(q, k, v, gv, beta, S0, scale=1.0, delta=True, chunk_size=8)
    assert torch.allclose(o1, o2, atol=1e-11) and torch.allclose(S1, S2, atol=1e-11)


def test_empty_and_no_initial_state():
    q, k, v, g, beta, _ = inputs(L=0)
    o, S = chunk_scan(q, k, v, g, beta, None, scale=1.0, delta=True, chunk_size=8)
    assert o.shape == (2, 0, 2, 6) and torch.count_nonzero(S) == 0
    q, k, v, g, beta, _ = inputs(L=5)
    o1, _ = recurrent_scan(q, k, v, g, beta, None, scale=1.0, delta=True)
    o2, _ = chunk_scan(q, k, v, g, beta, None, scale=1.0, delta=True, chunk_size=8)
    assert torch.allclose(o1, o2, atol=1e-12)


def test_asymmetric_write_matches_recurrence():
    q, k, v, g, _, S0 = inputs(gate="vector")
    w = 0.3 * torch.randn_like(k)
    o_r, S_r = recurrent_scan(q, k, v, g, None, S0, scale=0.7, delta=True, w=w)
    for C in (4, 8, 16):
        o_c, S_c = chunk_scan_vec(q, k, v, g, None, S0, scale=0.7, delta=True, chunk_size=C, w=w)
        assert torch.allclose(o_c, o_r, atol=1e-10) and torch.allclose(S_c, S_r, atol=1e-10)


def test_residual_scan_ratio():
    q, k, v, g, beta, _ = inputs()
    r = residual_scan(k, v, g, beta, None, delta=True)
    assert r.shape == (2, 37, 2) and torch.allclose(r[:, 0], torch.ones_like(r[:, 0]).float())
    assert torch.all(residual_scan(k, v, g, beta, None, delta=False) == 1)


def test_flops_and_fusions():
    assert chunk_scan_flops(16, 32, 8, True) == 3 * (6 * 16 * 32 + 2 * 8 * (3 * 16 + 2 * 32))
    assert chunk_scan_flops(16, 32, 8, False) == 3 * (4 * 16 * 32 + 2 * 8 * (16 + 32))
    assert parse_fusions("scan") == {"l2norm", "gate", "beta"}
    assert parse_fusions(True) == frozenset(("conv", "l2norm", "gate", "beta", "norm_gate"))
    assert parse_fusions(None) == frozenset()
    with pytest.raises(AssertionError):
        parse_fusions("bogus")


def _layer(gate="vector", **kw):
    torch.manual_seed(0)
    return GatedDeltaNet(32, 2, 8, 16, gate=gate, gate_rank=8, chunk_size=8, impl="torch", **kw).double()


@pytest.mark.parametrize("gate", ["none", "scalar", "vector"])
def test_module_decode_matches_forward(gate):
    m = _layer(gate)
    x = torch.randn(2, 21, 32, dtype=torch.float64)
    ref = m(x)
    m.reset_cache(2, 64)
    outs = [m.decode_step(x[:, :9])]
    snap = m.export_cache()
    outs += [m.decode_step(x[:, t:t + 1]) for t in range(9, 14)]
    outs.append(m.decode_step(x[:, 14:]))
    assert torch.allclose(torch.cat(outs, 1), ref, atol=1e-10)
    m2 = _layer(gate)
    m2.load_state_dict(m.state_dict())
    m2.load_cache(snap)
    assert torch.allclose(m2.decode_step(x[:, 9:]), ref[:, 9:], atol=1e-10)
    assert m.decode_step(x[:, :0]).shape[1] == 0


def test_causality_and_all_params_get_grads():
    m = _layer()
    x = torch.randn(1, 16, 32, dtype=torch.float64, requires_grad=True)
    y = m(x)
    y[:, 7].sum().backward()
    assert torch.all(x.grad[:, 8:] == 0) and torch.any(x.grad[:, :8] != 0)
    m.zero_grad()
    m(torch.randn(2, 16, 32, dtype=torch.float64)).sum().backward()
    assert all(p.grad is not None for p in m.parameters())


def test_gate_init_and_stats():
    m = _layer("vector", A_init_range=(1.0, 16.0))
    A = m.A_log.exp()
    assert torch.all(A >= 1 - 1e-6) and torch.all(A <= 16 + 1e-6)
    dt = F.softplus(m.dt_bias)
    assert torch.all(dt >= 1e-4) and torch.all(dt <= 0.1 + 1e-6)
    st = m.gate_stats(torch.randn(1, 16, 32, dtype=torch.float64))
    assert set(st) == {"state_rms", "alpha", "mem_len", "beta"}
    assert torch.all((st["alpha"] > 0) & (st["alpha"] < 1))
    b = _layer("vector", gate_lower_bound=-5.0)
    a = b.gate_stats(torch.zeros(1, 8, 32, dtype=torch.float64))["alpha"]
    assert torch.all(a < 1.0 - 1e-4), "the bounded gate must start with real forgetting"


def test_shortconv_shift_matches_conv1d():
    torch.manual_seed(0)
    c1 = ShortConv(12, 4, impl="conv1d").double()
    c2 = ShortConv(12, 4, impl="shift").double()
    c2.load_state_dict(c1.state_dict())
    x1 = torch.randn(2, 9, 12, dtype=torch.float64, requires_grad=True)
    x2 = x1.detach().clone().requires_grad_(True)
    y1, y2 = c1(x1, "silu"), c2(x2, "silu")
    assert torch.allclose(y1, y2, atol=1e-12)
    y1.sum().backward()
    y2.sum().backward()
    assert torch.allclose(x1.grad, x2.grad, atol=1e-12)
    assert torch.allclose(c1.conv.weight.grad, c2.conv.weight.grad, atol=1e-12)


def test_kda_intra_stage_matches_vector_oracle():
    """The per-channel-gate intra stage of ops/kda.py (its CPU path: gated
    products on 16-row sub-chunks) followed by the chunk recurrence
    V' = U - W S, O = Qh S + A V', S <- diag(gamma) S + Kt^T V' equals the
    pairwise-decay oracle chunk_scan_vec."""
    from vagus_b200.ops.kda import _gated, kda_intra
    torch.manual_seed(0)
    B, L, H, dk, dv = 1, 128, 2, 16, 8
    q = F.normalize(torch.randn(B, L, H, dk, dtype=torch.float64), dim=-1)
    k = F.normalize(torch.randn(B, L, H, dk, dtype=torch.float64), dim=-1)
    v = torch.randn(B, L, H, dv, dtype=torch.float64)
    g = F.logsigmoid(torch.randn(B, L, H, dk, dtype=torch.float64) + 2) * 0.5
    beta = torch.sigmoid(torch.randn(B, L, H, dtype=torch.float64))
    S0 = 0.1 * torch.randn(B, H, dk, dv, dtype=torch.float64)
    scale = dk ** -0.5
    o_r, S_r = chunk_scan_vec(q, k, v, g, beta, S0, scale=scale, delta=True, chunk_size=64)
    W, Qh, Kt, A, U, gam = kda_intra(q, k, v, g, beta, scale)
    S = S0.float()
    outs = []
    for n in range(L // 64):
        Vp = U[:, :, n] - W[:, :, n] @ S
        outs.append(Qh[:, :, n] @ S + A[:, :, n] @ Vp)
        S = gam[:, :, n, :, None] * S + Kt[:, :, n].transpose(-1, -2) @ Vp
    o = torch.stack(outs, 2).permute(0, 2, 3, 1, 4).reshape(B, L, H, dv)
    assert (o - o_r.float()).abs().max() < 1e-5 and (S - S_r.float()).abs().max() < 1e-5
    # the asymmetric write (an explicit write vector w, beta unused) on the same recurrence
    w = 0.5 * torch.rand(B, L, H, dk, dtype=torch.float64) * k
    o_r, S_r = chunk_scan_vec(q, k, v, g, None, S0, scale=scale, delta=True, chunk_size=64, w=w)
    W, Qh, Kt, A, U, gam = kda_intra(q, k, v, g, None, scale, w=w)
    S = S0.float()
    outs = []
    for n in range(L // 64):
        Vp = U[:, :, n] - W[:, :, n] @ S
        outs.append(Qh[:, :, n] @ S + A[:, :, n] @ Vp)
        S = gam[:, :, n, :, None] * S + Kt[:, :, n].transpose(-1, -2) @ Vp
    o = torch.stack(outs, 2).permute(0, 2, 3, 1, 4).reshape(B, L, H, dv)
    assert (o - o_r.float()).abs().max() < 1e-5 and (S - S_r.float()).abs().max() < 1e-5
    # gated linear attention (no delta rule): W = 0 and U = V on the same recurrence
    o_r, S_r = chunk_scan_vec(q, k, v, g, None, S0, scale=scale, delta=False, chunk_size=64)
    W, Qh, Kt, A, U, gam = kda_intra(q, k, v, g, beta, scale, delta=False)
    assert torch.count_nonzero(W) == 0
    S = S0.float()
    outs = []
    for n in range(L // 64):
        Vp = U[:, :, n] - W[:, :, n] @ S
        outs.append(Qh[:, :, n] @ S + A[:, :, n] @ Vp)
        S = gam[:, :, n, :, None] * S + Kt[:, :, n].transpose(-1, -2) @ Vp
    o = torch.stack(outs, 2).permute(0, 2, 3, 1, 4).reshape(B, L, H, dv)
    assert (o - o_r.float()).abs().max() < 1e-5 and (S - S_r.float()).abs().max() < 1e-5
    # the sub-chunk factorisation equals the pairwise definition, also for fast channels
    X, Y = torch.randn(2, 64, 8, dtype=torch.float64), torch.randn(2, 64, 8, dtype=torch.float64)
    gg = (-torch.rand(2, 64, 8, dtype=torch.float64) * 6).cumsum(-2)
    for strict in (True, False):
        E = (gg[..., :, None, :] - gg[..., None, :, :])
        mask = torch.ones(64, 64, dtype=torch.bool).tril(-1 if strict else 0)
        ref = torch.einsum("...ic,...ijc,...jc->...ij", X, E.masked_fill(~mask[..., None], float("-inf")).exp(), Y)
        assert torch.allclose(_gated(X, Y, gg, strict), ref, atol=1e-12)
