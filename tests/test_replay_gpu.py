"""Run-twice replay: every kernel whose reduction order is fixed must give
bit-identical outputs on identical inputs.  This is the determinism half of
the race-detection substitute (a race between threads or CTAs shows up as a
run-to-run difference long before it shows up as a wrong answer).

Exempt, by design -- their floating-point sums depend on arrival order:
  * GEMMs in atomic mode (split-K / stream-K weight gradients: fp32 red.add),
    and so the weight gradient of the fused cross-entropy;
  * the short-conv weight gradient (per-CTA partial sums combined with atomics);
  * the RMSNorm gain gradient (per-CTA row sums combined with atomics);
  * the attention backward's dQ (bulk tensor reduce-add of per-key-block
    partials);
  * gradients of the gated delta rule's per-sequence inputs that are summed
    over chunks with atomics (the initial state, the gates).
Everything else is compared with torch.equal."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _twice(fn):
    torch.manual_seed(0)
    a = fn()
    torch.cuda.synchronize()
    b = fn()
    torch.cuda.synchronize()
    a = a if isinstance(a, (tuple, list)) else (a,)
    b = b if isinstance(b, (tuple, list)) else (b,)
    return a, b


def _same(a, b, names):
    for n, x, y in zip(names, a, b):
        if x is None:
            continue
        assert torch.equal(x, y), f"{n}: max |diff| {(x.float() - y.float()).abs().max().item()}"


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(1024, 4160, 1024), (304, 328, 200)])
def test_gemm_store_mode_replays(a_mn, b_mn, M, N, K):
    from vagus_b200.ops import native
    g = torch.Generator(device=DEV).manual_seed(1)
    A = torch.randn((K, M) if a_mn else (M, K), device=DEV, generator=g).bfloat16()
    B = torch.randn((K, N) if b_mn else (N, K), device=DEV, generator=g).bfloat16()

    def run():
        C = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        assert native().gemm(A, a_mn, B, b_mn, C, None, 1.0, 0.0, False, 0, 0) == 0
        return C
    a, b = _twice(run)
    _same(a, b, ["C"])


def test_norm_swiglu_replay():
    from vagus_b200 import ops
    from vagus_b200.ops import native
    x = torch.randn(4096, 1024, device=DEV).requires_grad_(True)
    w = torch.rand(1024, device=DEV).requires_grad_(True)
    dy = torch.randn(4096, 1024, device=DEV)

    def run():
        xx, ww = x.detach().clone().requires_grad_(True), w.detach().clone().requires_grad_(True)
        y = ops.rmsnorm(xx, ww, 1e-6)
        y.backward(dy.to(y.dtype))
        return y, xx.grad
    a, b = _twice(run)
    _same(a, b, ["y", "dx"])
    u = torch.randn(4096, 2 * 2816, device=DEV).bfloat16()
    ds = torch.randn(4096, 2816, device=DEV).bfloat16()

    def run_sw():
        return native().swiglu_fwd(u), native().swiglu_bwd(ds, u)
    a, b = _twice(run_sw)
    _same(a, b, ["s", "du"])


def test_conv_forward_and_input_gradient_replay():
    from vagus_b200.ops import native
    B, L, D, K, hd = 2, 1000, 512, 4, 256
    x = torch.randn(B, L, D, device=DEV).bfloat16()
    w = 0.3 * torch.randn(D, 1, K, device=DEV)
    dy = torch.randn(B, L, D, device=DEV).bfloat16()

    def run():
        y, rn = native().conv_silu_fwd(x, w, hd, True)
        dx = torch.zeros(B, L, D, device=DEV, dtype=torch.bfloat16)
        dw = torch.zeros(D * K, device=DEV)
        native().conv_silu_bwd(dy, x, w, rn, dx, dw, hd, True)
        return y, dx
    a, b = _twice(run)
    _same(a, b, ["y", "dx"])


def test_gated_delta_rule_replay():
    from vagus_b200 import ops
    Bs, L, H, dk, dv = 2, 512, 2, 256, 256
    q = F.normalize(torch.randn(Bs, L, H, dk, device=DEV), dim=-1).bfloat16()
    k = F.normalize(torch.randn(Bs, L, H, dk, device=DEV), dim=-1).bfloat16()
    v = torch.randn(Bs, L, H, dv, device=DEV).bfloat16()
    g = F.logsigmoid(torch.randn(Bs, L, H, device=DEV) + 3)
    beta = torch.sigmoid(torch.randn(Bs, L, H, device=DEV))
    do = torch.randn(Bs, L, H, dv, device=DEV).bfloat16()

    def run():
        leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
        o, S = ops.gdr_chunk(*leaves, g, beta, None, scale=dk ** -0.5)
        o.backward(do)
        return (o, S) + tuple(t.grad for t in leaves)
    a, b = _twice(run)
    _same(a, b, ["o", "S", "dq", "dk", "dv"])


def test_attention_forward_and_kv_gradients_replay():
    from vagus_b200.ops.attention import attention
    B, H, L, D = 2, 4, 1024, 64
    q = torch.randn(B, H, L, D, device=DEV).bfloat16()
    k = torch.randn(B, H, L, D, device=DEV).bfloat16()
    v = torch.randn(B, H, L, D, device=DEV).bfloat16()
    do = torch.randn(B, H, L, D, device=DEV).bfloat16()

    def run():
        leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
        o = attention(*leaves, True)
        o.backward(do)
        return o, leaves[1].grad, leaves[2].grad
    a, b = _twice(run)
    _same(a, b, ["o", "dk", "dv"])


def test_mobius_scan_replay():
    from vagus_b200 import ops
    shp = (2, 2048, 4, 16)
    g = torch.Generator(device=DEV).manual_seed(3)
    m = 2.0 * torch.rand(shp, device=DEV, generator=g)
    w = 0.05 + torch.rand(shp, device=DEV, generator=g)
    a0 = 0.5 + 0.5 * torch.rand(shp, device=DEV, generator=g)
    coeffs = [1.0 + m * w, m * a0, w, a0]
    x0 = 0.5 + torch.rand((2, 4, 16), device=DEV, generator=g)
    gO = torch.randn(shp, device=DEV, generator=g)

    def run():
        leaves = [t.clone().requires_grad_(True) for t in coeffs + [x0]]
        out = ops.mobius_scan(*leaves)
        out.backward(gO)
        return (out,) + tuple(t.grad for t in leaves)
    a, b = _twice(run)
    _same(a, b, ["x", "dA", "dB", "dC", "dD", "dx0"])
