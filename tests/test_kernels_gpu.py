# Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of
# the same op, on small shapes that still cover tails and every layout.
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _g(*args):
    from vagus_b200.ops import native
    rc = native().gemm(*args)
    assert rc == 0, rc


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield
    from vagus_b200 import ops
    torch.cuda.synchronize()
    ops.check_error()


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (200, 328, 136), (1024, 4104, 1024), (384, 128, 64)])
def test_gemm_layouts(a_mn, b_mn, M, N, K):
    from vagus_b200.ops import native
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    Ast = A.t().contiguous() if a_mn else A
    Bst = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    C = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    _g(Ast, a_mn, Bst, b_mn, C, None, 1.0, 0.0, False, 0, 0)
    assert rel(C, ref) < 1e-2
    C32 = torch.empty(M, N, device=DEV, dtype=torch.float32)
    _g(Ast, a_mn, Bst, b_mn, C32, None, 1.0, 0.0, False, 0, 0)
    assert rel(C32, ref) < 2e-3


def test_gemm_rejects_boxes_larger_than_tensor():
    from vagus_b200.ops import native
    A = torch.randn(64, 64, device=DEV).bfloat16()
    B = torch.randn(8, 64, device=DEV).bfloat16()
    C = torch.empty(64, 8, device=DEV, dtype=torch.bfloat16)
    assert native().gemm(A, False, B, False, C, None, 1.0, 0.0, False, 0, 0) == 6
    from vagus_b200.ops._core import gemm
    with pytest.raises(RuntimeError):
        gemm(A, False, B, False, C)


def test_gemm_epilogues_and_batch():
    from vagus_b200.ops import native
    M, N, K, Bt = 384, 640, 320, 3
    A = torch.randn(Bt, M, K, device=DEV).bfloat16()
    B = torch.randn(Bt, N, K, device=DEV).bfloat16()
    S = torch.randn(Bt, M, N, device=DEV)
    ref = 0.5 * (A.float() @ B.float().transpose(1, 2)) - 2.0 * S
    C = torch.empty(Bt, M, N, device=DEV)
    _g(A, False, B, False, C, S, 0.5, -2.0, False, 0, 0)
    assert rel(C, ref) < 2e-3
    # atomic split-K accumulation into an fp32 buffer (weight-gradient shape)
    T, Dout, Din = 4096, 256, 512
    dy = torch.randn(T, Dout, device=DEV).bfloat16()
    x = torch.randn(T, Din, device=DEV).bfloat16()
    acc = torch.randn(Dout, Din, device=DEV)
    ref = acc + dy.float().t() @ x.float()
    _g(dy, True, x, True, acc, None, 1.0, 0.0, True, 0, 0)
    assert rel(acc, ref) < 2e-3
    for bn in (128, 256):
        C = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        _g(A[0], False, B[0], False, C, None, 1.0, 0.0, False, 1, bn)
        assert rel(C, A[0].float() @ B[0].float().t()) < 1e-2


def test_linear_autograd():
    from vagus_b200 import ops
    x = torch.randn(3, 100, 256, device=DEV, requires_grad=True)
    w = torch.randn(384, 256, device=DEV, requires_grad=True)
    r = torch.randn(3, 100, 384, device=DEV, requires_grad=True)
    y = ops.linear_residual(r, x.bfloat16(), w)
    xr, wr, rr = (t.detach().clone().requires_grad_(True) for t in (x, w, r))
    yr = rr + xr.bfloat16().float() @ wr.bfloat16().float().t()
    g = torch.randn_like(yr)
    (y * g).sum().backward()
    (yr * g).sum().backward()
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 1e-2 and rel(w.grad, wr.grad) < 1e-2 and rel(r.grad, rr.grad) < 1e-6


@pytest.mark.parametrize("xdt,odt", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float32, torch.float32)])
def test_rmsnorm(xdt, odt):
    from vagus_b200 import ops
    x = torch.randn(333, 1024, device=DEV, dtype=xdt, requires_grad=True)
    g = (1 + 0.1 * torch.randn(1024, device=DEV)).requires_grad_(True)
    y = ops.rmsnorm(x, g, 1e-6, out_dtype=odt)
    xr, gr = x.detach().float().requires_grad_(True), g.detach().clone().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * gr
    dy = torch.randn_like(yr)
    (y.float() * dy).sum().backward()
    (yr * dy).sum().backward()
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 1e-2 and rel(g.grad, gr.grad) < 1e-2


def test_rmsnorm_gated_and_swiglu_and_sgate():
    from vagus_b200 import ops
    o = torch.randn(50, 4, 256, device=DEV).bfloat16().requires_grad_(True)
    gt = torch.randn(50, 4, 256, device=DEV).bfloat16().requires_grad_(True)
    gm = (1 + 0.1 * torch.randn(256, device=DEV)).requires_grad_(True)
    y = ops.rmsnorm_gated(o, gt, gm, 1e-6)
    orr, gr, gmr = (t.detach().float().requires_grad_(True) for t in (o, gt, gm))
    yr = orr * torch.rsqrt(orr.pow(2).mean(-1, keepdim=True) + 1e-6) * gmr * F.silu(gr)
    dy = torch.randn_like(yr)
    (y.float() * dy).sum().backward()
    (yr * dy).sum().backward()
    assert rel(y, yr) < 1e-2
    for a, b in ((o, orr), (gt, gr), (gm, gmr)):
        assert rel(a.grad, b.grad) < 2e-2
    u = torch.randn(77, 2 * 704, device=DEV).bfloat16().requires_grad_(True)
    s = ops.swiglu(u)
    ur = u.detach().float().requires_grad_(True)
    a, b = ur.chunk(2, -1)
    sr = F.silu(a) * b
    ds = torch.randn_like(sr)
    (s.float() * ds).sum().backward()
    (sr * ds).sum().backward()
    assert rel(s, sr) < 1e-2 and rel(u.grad, ur.grad) < 1e-2
    xx = torch.randn(1000, device=DEV).bfloat16().requires_grad_(True)
    gg = torch.randn(1000, device=DEV).bfloat16().requires_grad_(True)
    z = ops.sigmoid_gate(xx, gg)
    xr2, gr2 = xx.detach().float().requires_grad_(True), gg.detach().float().requires_grad_(True)
    zr = xr2 * torch.sigmoid(gr2)
    dz = torch.randn_like(zr)
    (z.float() * dz).sum().backward()
    (zr * dz).sum().backward()
    assert rel(z, zr) < 1e-2 and rel(xx.grad, xr2.grad) < 1e-2 and rel(gg.grad, gr2.grad) < 1e-2


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("norm,rope", [(True, True), (False, True), (True, False)])
def test_qk_norm_rope(norm, rope, D):
    """qk-norm + RoPE (vectorised kernels at head dims 64 / 128; 222 rows, not
    a multiple of the rows a warp covers) against fp32 torch, incl. gradients."""
    from vagus_b200 import ops
    from vagus_b200.models.rope import RoPE
    B, L, H = 2, 37, 3
    x = torch.randn(B, L, H, D, device=DEV).bfloat16().requires_grad_(True)
    gm = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_(True) if norm else None
    rp = RoPE(H * D, D, 64).to(DEV)
    tables = rp.tables(L, 5) if rope else None
    y = ops.qk_norm_rope(x, gm, tables, 1e-6)
    xr = x.detach().float().requires_grad_(True)
    gr = gm.detach().clone().requires_grad_(True) if norm else None
    h = xr
    if norm:
        h = (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)) * gr
    if rope:
        h = rp(h.transpose(1, 2), 5).transpose(1, 2)
    dy = torch.randn_like(h)
    (y.float() * dy).sum().backward()
    (h * dy).sum().backward()
    assert rel(y, h) < 1e-2 and rel(x.grad, xr.grad) < 2e-2
    if norm:
        assert rel(gm.grad, gr.grad) < 2e-2


def test_qk_norm_rope_pitched():
    """The RoPE kernels on a column slice of a packed projection (token pitch
    wider than the heads), writing the input gradient into a slice of a packed
    gradient: same values as on dense copies."""
    from vagus_b200.ops import native
    from vagus_b200.models.rope import RoPE
    B, L, H, D, NP, c0 = 2, 45, 3, 64, 512, 128
    P = torch.randn(B, L, NP, device=DEV).bfloat16()
    x = P[:, :, c0:c0 + H * D].view(B, L, H, D)
    gm = 1 + 0.1 * torch.randn(D, device=DEV)
    cos, sin = (t.float().contiguous() for t in RoPE(H * D, D, 64).to(DEV).tables(L, 3))
    C = native()
    y, rs = C.qk_norm_rope_fwd(x, gm, cos, sin, 1e-6)
    y0, rs0 = C.qk_norm_rope_fwd(x.contiguous(), gm, cos, sin, 1e-6)
    assert torch.equal(y, y0) and torch.equal(rs, rs0)
    dy = torch.randn(B, L, H, D, device=DEV).bfloat16()
    dP = torch.zeros(B, L, NP, device=DEV, dtype=torch.bfloat16)
    dx_slice = dP[:, :, c0:c0 + H * D].view(B, L, H, D)
    _, dg = C.qk_norm_rope_bwd(dy, x, gm, cos, sin, rs, dx_slice)
    dx0, dg0 = C.qk_norm_rope_bwd(dy, x.contiguous(), gm, cos, sin, rs0)
    assert torch.equal(dx_slice, dx0) and rel(dg, dg0) < 1e-5
    assert dP[:, :, :c0].abs().sum() == 0 and dP[:, :, c0 + H * D:].abs().sum() == 0


@pytest.mark.parametrize("H,Hk,D,vm,rope,qkn", [(8, 8, 64, 1, True, False), (4, 2, 128, 1, True, False),
                                                  (4, 2, 128, 1, True, True), (4, 2, 64, 2, True, False),
                                                  (4, 2, 64, 2, False, False), (4, 4, 64, 1, False, True)])
def test_attention_layer_fused_matches_fp32(H, Hk, D, vm, rope, qkn):
    """The fused layer (q / k / v packed into one GEMM, RoPE on slices of it,
    attention reading v out of it, one dgrad and one wgrad GEMM; with RoPE
    alone the attention backward un-rotates dq / dk itself) against the same
    module run unfused in fp32: output, input gradient, every weight gradient
    and the qk-norm gains."""
    from vagus_b200 import ops
    from vagus_b200.models.attention import SoftmaxAttention
    from vagus_b200.models.rope import RoPE
    B, L, dim = 2, 256, H * D
    m = SoftmaxAttention(dim, H, Hk, vm, qk_norm=qkn, rope=RoPE(dim, D, L) if rope else None).to(DEV)
    if qkn:
        with torch.no_grad():
            m.q_norm.gamma.add_(0.1 * torch.randn_like(m.q_norm.gamma))
            m.k_norm.gamma.add_(0.1 * torch.randn_like(m.k_norm.gamma))
    x = torch.randn(B, L, dim, device=DEV)
    xb = x.bfloat16().requires_grad_(True)
    assert ops.attention_layer_ok(m, xb)
    y = m.forward_pre_out(xb)
    dy = torch.randn_like(y, dtype=torch.float32)
    (y.float() * dy).sum().backward()
    got = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
    m.zero_grad()
    xr = x.clone().requires_grad_(True)
    assert not ops.attention_layer_ok(m, xr)
    yr = m.forward_pre_out(xr)
    (yr * dy).sum().backward()
    assert rel(y, yr) < 2e-2 and rel(xb.grad, xr.grad) < 3e-2
    ref = {n: p.grad for n, p in m.named_parameters() if p.grad is not None}
    assert set(got) == set(ref) and {"wq.weight", "wk.weight", "wv.weight"} <= set(got)
    for n, g in ref.items():
        assert rel(got[n], g) < 3e-2, n


def test_transformerpp_bf16_matches_cpu_fp32():
    """A small Transformer++ (head dim 64, fused attention layers, SwiGLU,
    fused CE) under bf16 autocast on the GPU against the same weights in fp32
    on the CPU: loss and every parameter gradient."""
    from vagus_b200.models import build_model
    from vagus_b200.models.losses import make_ce
    args = dict(vocab_size=2048, dim=256, head_dim=64, context_len=512, layer_count=2, ffn_hidden_dim=704)
    model = build_model("TransformerPP", args).to(DEV)
    ref = build_model("TransformerPP", args)
    ref.load_state_dict({k: v.detach().cpu() for k, v in model.state_dict().items()})
    tok = torch.randint(0, 2048, (2, 257), device=DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = make_ce("fused")(model(tok[:, :-1], return_hidden=True), model.head.weight, tok[:, 1:])
    loss.backward()
    tc = tok.cpu()
    loss_ref = make_ce("full")(ref(tc[:, :-1], return_hidden=True), ref.head.weight, tc[:, 1:])
    loss_ref.backward()
    assert abs(loss.item() - loss_ref.item()) <= 1e-2 * abs(loss_ref.item())
    got = dict(model.named_parameters())
    for n, p in ref.named_parameters():
        assert rel(got[n].grad.cpu(), p.grad) < 5e-2, n


def _conv_ref(x, w, hd, l2):
    D, K = w.shape[0], w.shape[-1]
    y = F.conv1d(F.pad(x.transpose(1, 2), (K - 1, 0)), w, groups=D).transpose(1, 2)
    z = F.silu(y)
    if l2:
        B, L = z.shape[:2]
        zz = z.view(B, L, D // hd, hd)
        z = (zz * torch.rsqrt(zz.pow(2).sum(-1, keepdim=True) + 1e-6)).view(B, L, D)
    return z


@pytest.mark.parametrize("l2", [True, False])
@pytest.mark.parametrize("L,hd", [(150, 256), (67, 128), (5, 256), (300, 64)])
def test_conv_silu(l2, L, hd):
    from vagus_b200.ops import native
    B, D, K = 2, 512, 4
    big = torch.randn(B, L, 3 * D, device=DEV).bfloat16()
    x = big[:, :, D:2 * D]
    w = 0.3 * torch.randn(D, 1, K, device=DEV)
    y, rn = native().conv_silu_fwd(x, w, hd, l2)
    xr = x.float().detach().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = _conv_ref(xr, wr, hd, l2)
    assert rel(y, yr) < 1e-2
    dy = torch.randn_like(yr)
    (yr * dy).sum().backward()
    dxbig = torch.zeros_like(big)
    dw = torch.zeros(D * K, device=DEV)
    native().conv_silu_bwd(dy.bfloat16(), x, w, rn, dxbig[:, :, D:2 * D], dw, hd, l2)
    assert rel(dxbig[:, :, D:2 * D], xr.grad) < 2e-2
    assert rel(dw.view(D, 1, K), wr.grad) < 2e-2
    assert dxbig[:, :, :D].abs().max().item() == 0


def test_gates():
    from vagus_b200.ops import native
    T, H = 300, 4
    ab = torch.randn(T, 2 * H, device=DEV).bfloat16()
    A_log = torch.rand(H, device=DEV).log1p()
    dtb = torch.randn(H, device=DEV)
    g, beta = native().gdn_gates_fwd(ab, A_log, dtb, H)
    abr = ab.float().requires_grad_(True)
    Ar, dr = A_log.clone().requires_grad_(True), dtb.clone().requires_grad_(True)
    gr = -Ar.exp() * F.softplus(abr[:, :H] + dr)
    br = torch.sigmoid(abr[:, H:])
    assert rel(g, gr) < 1e-4 and rel(beta, br) < 1e-4
    dg, db = torch.randn_like(gr), torch.randn_like(br)
    ((gr * dg).sum() + (br * db).sum()).backward()
    dab = torch.empty_like(ab)
    dA, ddt = native().gdn_gates_bwd(dg, db, ab, A_log, dtb, H, dab)
    assert rel(dab, abr.grad) < 1e-2 and rel(dA, Ar.grad) < 1e-4 and rel(ddt, dr.grad) < 1e-4


def _gdr_inputs(B, L, H, dk, dv):
    q = F.normalize(torch.randn(B, L, H, dk, device=DEV), dim=-1)
    k = F.normalize(torch.randn(B, L, H, dk, device=DEV), dim=-1)
    v = torch.randn(B, L, H, dv, device=DEV)
    g = F.logsigmoid(torch.randn(B, L, H, device=DEV) + 3)
    beta = torch.sigmoid(torch.randn(B, L, H, device=DEV))
    return q, k, v, g, beta


@pytest.mark.parametrize("dk,dv", [(128, 128), (256, 256), (128, 256)])
def test_gdr_chunk_fwd_bwd(dk, dv):
    from vagus_b200 import ops
    from vagus_b200.models.scans import chunk_scan
    B, L, H = 2, 200, 2
    q, k, v, g, beta = _gdr_inputs(B, L, H, dk, dv)
    S0 = 0.1 * torch.randn(B, H, dk, dv, device=DEV)
    scale = dk ** -0.5
    ins = [t.bfloat16().float() for t in (q, k, v)] + [g, beta, S0]
    ref_in = [t.clone().requires_grad_(True) for t in ins]
    o_r, S_r = chunk_scan(*ref_in[:5], ref_in[5], scale=scale, delta=True, chunk_size=64)
    cu_in = [t.clone().requires_grad_(True) for t in ins]
    o, S = ops.gdr_chunk(cu_in[0].bfloat16(), cu_in[1].bfloat16(), cu_in[2].bfloat16(), cu_in[3], cu_in[4],
                         cu_in[5], scale=scale)
    assert rel(o, o_r) < 2e-2 and rel(S, S_r) < 2e-2
    do, dS = torch.randn_like(o_r), torch.randn_like(S_r)
    ((o_r * do).sum() + (S_r * dS).sum()).backward()
    ((o.float() * do).sum() + (S * dS).sum()).backward()
    for a, b in zip(cu_in, ref_in):
        assert rel(a.grad, b.grad) < 5e-2, (a.shape, rel(a.grad, b.grad))


@pytest.mark.parametrize("dk,dv,L", [(128, 256, 200), (128, 128, 256)])
def test_kda_chunk_fwd_bwd(dk, dv, L):
    """Per-channel gate (KDA): torch intra stage + recurrence kernels vs the
    fp32 chunk oracle, outputs, final state and every input gradient."""
    from vagus_b200 import ops
    from vagus_b200.models.scans import chunk_scan_vec
    B, H = 2, 2
    q, k, v, _, beta = _gdr_inputs(B, L, H, dk, dv)
    g = F.logsigmoid(torch.randn(B, L, H, dk, device=DEV) + 2) * 0.5
    S0 = 0.1 * torch.randn(B, H, dk, dv, device=DEV)
    scale = dk ** -0.5
    ins = [t.bfloat16().float() for t in (q, k, v)] + [g, beta, S0]
    ref_in = [t.clone().requires_grad_(True) for t in ins]
    o_r, S_r = chunk_scan_vec(ref_in[0], ref_in[1], ref_in[2], ref_in[3], ref_in[4], ref_in[5], scale=scale,
                              delta=True, chunk_size=64)
    cu_in = [t.clone().requires_grad_(True) for t in ins]
    o, S = ops.kda_chunk(cu_in[0].bfloat16(), cu_in[1].bfloat16(), cu_in[2].bfloat16(), cu_in[3], cu_in[4],
                         cu_in[5], scale=scale)
    assert rel(o, o_r) < 2e-2 and rel(S, S_r) < 2e-2, (rel(o, o_r), rel(S, S_r))
    do, dS = torch.randn_like(o_r), torch.randn_like(S_r)
    ((o_r * do).sum() + (S_r * dS).sum()).backward()
    ((o.float() * do).sum() + (S * dS).sum()).backward()
    for name, a, b in zip("q k v g beta S0".split(), cu_in, ref_in):
        assert rel(a.grad, b.grad) < 5e-2, (name, rel(a.grad, b.grad))


@pytest.mark.parametrize("dv", [128, 256])
def test_kda_intra_kernels_match_fp32_oracle(dv):
    """The fused KDA intra-chunk kernels (per-channel cumulative decay, gated
    products, WY transform; and their backward) against the torch intra stage
    run in fp32 on the CPU (plain gated products and triangular solve)."""
    from vagus_b200.ops import native
    from vagus_b200.ops.kda import kda_intra
    B, L, H, dk = 2, 192, 2, 128
    q, k, v, _, beta = _gdr_inputs(B, L, H, dk, dv)
    g = F.logsigmoid(torch.randn(B, L, H, dk, device=DEV) + 2) * 0.5
    q, k, v = (t.bfloat16() for t in (q, k, v))
    scale = dk ** -0.5
    outs = native().kda_intra_fwd(q, k, v, g.contiguous(), beta.contiguous(), scale)
    ins = [t.float().cpu().requires_grad_(True) for t in (q, k, v, g, beta)]
    ref = kda_intra(*ins, scale)
    for name, a, r in zip(("W", "Qh", "Kt", "A", "U", "gC"), outs, ref):
        assert rel(a.float().cpu().view(r.shape), r.detach()) < 1e-2, (name, rel(a.float().cpu().view(r.shape), r))
    gen = torch.Generator().manual_seed(3)
    ups = [torch.randn(r.shape, generator=gen).bfloat16().float() for r in ref]
    sum(((r * u).sum() for r, u in zip(ref, ups))).backward()
    flat = lambda t: t.reshape(B * H, L // 64, *t.shape[3:]).contiguous().to(DEV)   # noqa: E731
    dW, dQh, dKt, dA, dU, dgC = (flat(u) for u in ups)
    grads = native().kda_intra_bwd(q, k, v, g.contiguous(), beta.contiguous(), dW.bfloat16(), dQh.bfloat16(),
                                   dKt.bfloat16(), dA, dU.bfloat16(), dgC, scale)
    for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta"), grads, ins):
        assert rel(a.float().cpu(), r.grad) < 2e-2, (name, rel(a.float().cpu(), r.grad))


def test_asymmetric_write_chunk_fwd_bwd():
    """An explicit write vector (the Kalman diagonal gain's asymmetric write)
    on the recurrence kernels vs the fp32 chunk oracle, incl. gradients."""
    from vagus_b200 import ops
    from vagus_b200.models.scans import chunk_scan_vec
    B, L, H, dk, dv = 2, 160, 2, 128, 128
    q, k, v, _, _ = _gdr_inputs(B, L, H, dk, dv)
    g = F.logsigmoid(torch.randn(B, L, H, dk, device=DEV) + 2) * 0.5
    w = 0.5 * torch.rand(B, L, H, dk, device=DEV) * k.float()
    S0 = 0.1 * torch.randn(B, H, dk, dv, device=DEV)
    scale = dk ** -0.5
    ins = [t.bfloat16().float() for t in (q, k, v)] + [g, w, S0]
    ref_in = [t.clone().requires_grad_(True) for t in ins]
    o_r, S_r = chunk_scan_vec(ref_in[0], ref_in[1], ref_in[2], ref_in[3], None, ref_in[5], scale=scale,
                              delta=True, chunk_size=64, w=ref_in[4])
    cu_in = [t.clone().requires_grad_(True) for t in ins]
    o, S = ops.kda_chunk(cu_in[0].bfloat16(), cu_in[1].bfloat16(), cu_in[2].bfloat16(), cu_in[3], None, cu_in[5],
                         scale=scale, w=cu_in[4])
    assert rel(o, o_r) < 2e-2 and rel(S, S_r) < 2e-2, (rel(o, o_r), rel(S, S_r))
    do, dS = torch.randn_like(o_r), torch.randn_like(S_r)
    ((o_r * do).sum() + (S_r * dS).sum()).backward()
    ((o.float() * do).sum() + (S * dS).sum()).backward()
    for name, a, b in zip("q k v g w S0".split(), cu_in, ref_in):
        assert rel(a.grad, b.grad) < 5e-2, (name, rel(a.grad, b.grad))


@pytest.mark.parametrize("gate,delta", [("scalar", False), ("vector", False), ("none", True), ("none", False)])
def test_gla_and_deltanet_chunk_fwd_bwd(gate, delta):
    """The other members of the family on the same kernels -- gated linear
    attention (no delta rule) and DeltaNet (no gate) -- against the fp32
    chunk oracle, outputs, final state and input gradients."""
    from vagus_b200 import ops
    from vagus_b200.models.scans import chunk_scan
    B, L, H, dk, dv = 2, 192, 2, 128, 128
    q, k, v, _, beta = _gdr_inputs(B, L, H, dk, dv)
    g = None
    if gate == "scalar":
        g = F.logsigmoid(torch.randn(B, L, H, device=DEV) + 2) * 0.5
    elif gate == "vector":
        g = F.logsigmoid(torch.randn(B, L, H, dk, device=DEV) + 2) * 0.5
    S0 = 0.1 * torch.randn(B, H, dk, dv, device=DEV)
    scale = dk ** -0.5
    ins = [t.bfloat16().float() for t in (q, k, v)] + [S0]
    ref_in = [t.clone().requires_grad_(True) for t in ins]
    o_r, S_r = chunk_scan(ref_in[0], ref_in[1], ref_in[2], g, beta if delta else None, ref_in[3], scale=scale,
                          delta=delta, chunk_size=64)
    cu_in = [t.clone().requires_grad_(True) for t in ins]
    o, S = ops.kda_chunk(cu_in[0].bfloat16(), cu_in[1].bfloat16(), cu_in[2].bfloat16(), g,
                         beta if delta else None, cu_in[3], scale=scale, delta=delta)
    assert rel(o, o_r) < 2e-2 and rel(S, S_r) < 2e-2, (rel(o, o_r), rel(S, S_r))
    do, dS = torch.randn_like(o_r), torch.randn_like(S_r)
    ((o_r * do).sum() + (S_r * dS).sum()).backward()
    ((o.float() * do).sum() + (S * dS).sum()).backward()
    for name, a, b in zip("q k v S0".split(), cu_in, ref_in):
        assert rel(a.grad, b.grad) < 5e-2, (name, rel(a.grad, b.grad))


@pytest.mark.parametrize("dk,dv", [(128, 128), (256, 256), (128, 256)])
def test_gdr_intra_kernel_matches_torch(dk, dv):
    from vagus_b200.ops import native
    from vagus_b200.ops.gdn import _intra
    B, L, H = 2, 192, 3
    q, k, v, g, beta = _gdr_inputs(B, L, H, dk, dv)
    q, k, v = (t.bfloat16() for t in (q, k, v))
    outs = native().gdr_intra_fwd(q, k, v, g, beta, 0.25)
    ref = _intra(q, k, v, g, beta, 0.25)
    for name, a, r in zip(("W", "Qh", "Kt", "A", "U", "gC"), outs, ref):
        assert rel(a.view(r.shape), r) < 2e-2, (name, rel(a.view(r.shape), r))


def test_gdr_decode():
    from vagus_b200 import ops
    from vagus_b200.models.scans import recurrent_scan
    B, H, dk, dv = 3, 2, 128, 64
    q, k, v, g, beta = _gdr_inputs(B, 1, H, dk, dv)
    S = torch.randn(B, H, dk, dv, device=DEV)
    o_r, S_r = recurrent_scan(q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float(), g, beta, S,
                              scale=0.3, delta=True)
    o, S2 = ops.gdr_decode(q.bfloat16(), k.bfloat16(), v.bfloat16(), g, beta, S, scale=0.3)
    assert rel(o, o_r) < 1e-2 and rel(S2, S_r) < 1e-4


def test_fused_linear_ce():
    from vagus_b200 import ops
    N, D, V = 1000, 256, 3000
    h = torch.randn(N, D, device=DEV).bfloat16().requires_grad_(True)
    w = (0.05 * torch.randn(V, D, device=DEV)).requires_grad_(True)
    t = torch.randint(0, V, (N,), device=DEV)
    loss, z = ops.fused_linear_ce(h, w, t, z_loss=1e-3)
    hr, wr = h.detach().float().requires_grad_(True), w.detach().clone().requires_grad_(True)
    lg = hr @ wr.bfloat16().float().t()
    zr = 1e-3 * torch.logsumexp(lg, -1).pow(2).mean()
    lr = F.cross_entropy(lg, t) + zr
    lr.backward()
    loss.backward()
    assert abs(loss.item() - lr.item()) < 2e-2 and abs(z.item() - zr.item()) < 1e-3
    assert rel(h.grad, hr.grad) < 3e-2 and rel(w.grad, wr.grad) < 3e-2


def test_embedding():
    from vagus_b200 import ops
    w = torch.randn(100, 64, device=DEV, requires_grad=True)
    t = torch.randint(0, 100, (4, 33), device=DEV)
    y = ops.embedding(t, w)
    wr = w.detach().clone().requires_grad_(True)
    yr = F.embedding(t, wr)
    dy = torch.randn_like(yr)
    (y * dy).sum().backward()
    (yr * dy).sum().backward()
    assert torch.equal(y, yr) and rel(w.grad, wr.grad) < 1e-5


def test_gdn_mixer_matches_torch_path():
    from vagus_b200.models.gdn import GatedDeltaNet
    torch.manual_seed(0)
    m = GatedDeltaNet(256, 2, 128, 128, gate="scalar", impl="cuda").to(DEV)
    m_ref = GatedDeltaNet(256, 2, 128, 128, gate="scalar", impl="torch").to(DEV)
    m_ref.load_state_dict(m.state_dict())
    x = torch.randn(2, 130, 256, device=DEV)
    xa = x.bfloat16().requires_grad_(True)
    y = m(xa)
    xb = x.bfloat16().float().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        yr = m_ref(xb)
    dy = torch.randn_like(yr.float())
    (y.float() * dy).sum().backward()
    (yr.float() * dy).sum().backward()
    assert rel(y, yr) < 3e-2
    assert rel(xa.grad, xb.grad) < 5e-2
    for (n, p), (_, pr) in zip(m.named_parameters(), m_ref.named_parameters()):
        assert rel(p.grad, pr.grad) < 8e-2, (n, rel(p.grad, pr.grad))


@pytest.mark.parametrize("dv", [128, 256])
def test_kda_mixer_matches_torch_path(dv):
    """The fused per-channel-gate layer (packed projection, KDA gate kernels,
    conv, fused KDA chunk, gated norm) against the same layer on the torch
    path (fp32 chunk oracle under bf16 autocast): output, input gradient and
    every parameter gradient."""
    from vagus_b200.models.gdn import GatedDeltaNet
    torch.manual_seed(0)
    m = GatedDeltaNet(256, 2, 128, dv, gate="vector", gate_rank=64, impl="cuda").to(DEV)
    m_ref = GatedDeltaNet(256, 2, 128, dv, gate="vector", gate_rank=64, impl="torch").to(DEV)
    m_ref.load_state_dict(m.state_dict())
    x = torch.randn(2, 130, 256, device=DEV)
    assert m._fused_kda_ok(x.bfloat16())
    xa = x.bfloat16().requires_grad_(True)
    y = m(xa)
    xb = x.bfloat16().float().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        yr = m_ref(xb)
    dy = torch.randn_like(yr.float())
    (y.float() * dy).sum().backward()
    (yr.float() * dy).sum().backward()
    assert rel(y, yr) < 3e-2, rel(y, yr)
    assert rel(xa.grad, xb.grad) < 5e-2, rel(xa.grad, xb.grad)
    for (n, p), (_, pr) in zip(m.named_parameters(), m_ref.named_parameters()):
        assert p.grad is not None and rel(p.grad, pr.grad) < 8e-2, (n, rel(p.grad, pr.grad))


def test_rmsnorm_pass_fuses_residual_gradient():
    """The (norm, identity) node adds both gradients in the norm kernel and
    hands the next linear_residual backward a bf16 copy; gradients match the
    plain composition."""
    from vagus_b200 import ops
    torch.manual_seed(0)
    T, D = 512, 1024
    x0 = torch.randn(T, D, device=DEV)
    gamma = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_(True)
    w = (0.02 * torch.randn(D, D, device=DEV)).requires_grad_(True)

    def run(fused):
        x = x0.clone().requires_grad_(True)
        norm = (lambda t: ops.rmsnorm_pass(t, gamma, 1e-6)) if fused else \
            (lambda t: (ops.rmsnorm(t, gamma, 1e-6, out_dtype=torch.bfloat16), t))
        h, xp = norm(x)
        y = ops.linear_residual(xp, h, w)
        h2, yp = norm(y)
        z = ops.linear_residual(yp, h2, w)
        (z.pow(2).sum() * 1e-3).backward()
        return x.grad.clone(), gamma.grad.clone(), w.grad.clone()

    ref = run(False)
    gamma.grad = None
    w.grad = None
    got = run(True)
    for a, b in zip(got, ref):
        assert rel(a, b) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 768, 384), (640, 392, 200), (296, 1000, 128)])
def test_gemm_cta_pair_matches_single_cta(a_mn, b_mn, M, N, K):
    """The CTA-pair kernel (block_n 512, 256 x 256 tiles over two SMs) and the
    one-CTA kernel (block_n 256) agree with the fp32 product, for stores and
    for split-K atomic accumulation."""
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    Ast = A.t().contiguous() if a_mn else A
    Bst = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    for bn in (512, 256):
        C = torch.empty(M, N, device=DEV, dtype=torch.float32)
        _g(Ast, a_mn, Bst, b_mn, C, None, 1.0, 0.0, False, 0, bn)
        assert rel(C, ref) < 2e-3, bn
        acc = torch.randn(M, N, device=DEV)
        want = acc + ref
        _g(Ast, a_mn, Bst, b_mn, acc, None, 1.0, 0.0, True, 0, bn)
        assert rel(acc, want) < 2e-3, bn


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H,Hk,Lq,Lk", [(4, 4, 256, 256), (4, 2, 200, 200), (2, 1, 100, 300)])
def test_flash_attention_fwd_bwd(D, causal, H, Hk, Lq, Lk):
    """sm_100a flash attention (forward + backward) against an fp32 softmax
    reference with lower-right causal alignment and GQA."""
    from vagus_b200.ops import native
    from vagus_b200.ops.attention import attention
    assert hasattr(native(), "attn_fwd")
    B = 2
    q = torch.randn(B, H, Lq, D, device=DEV).bfloat16().requires_grad_(True)
    k = torch.randn(B, Hk, Lk, D, device=DEV).bfloat16().requires_grad_(True)
    v = torch.randn(B, Hk, Lk, D, device=DEV).bfloat16().requires_grad_(True)
    o = attention(q, k, v, causal)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    rep = H // Hk
    kr, vr = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    s = (qf @ kr.transpose(-1, -2)) / math.sqrt(D)
    if causal:
        i = torch.arange(Lq, device=DEV)[:, None] + (Lk - Lq)
        j = torch.arange(Lk, device=DEV)[None, :]
        s = s.masked_fill(j > i, float("-inf"))
    ref = torch.softmax(s, -1) @ vr
    assert rel(o, ref) < 1e-2
    g = torch.randn_like(ref)
    (o.float() * g).sum().backward()
    (ref * g).sum().backward()
    assert rel(q.grad, qf.grad) < 2e-2
    assert rel(k.grad, kf.grad) < 2e-2
    assert rel(v.grad, vf.grad) < 2e-2


@pytest.mark.parametrize("D", [512, 1024, 2048])
def test_rmsnorm_backward_wide_rows(D):
    """The vectorised residual-stream backward (register and shared-memory
    gamma-partial variants) against the fp32 autograd reference."""
    from vagus_b200.ops import native
    T = 1000
    x = torch.randn(T, D, device=DEV)
    gamma = 1 + 0.1 * torch.randn(D, device=DEV)
    dy = torch.randn(T, D, device=DEV).bfloat16()
    dres = torch.randn(T, D, device=DEV)
    y, rstd = native().rmsnorm_fwd(x, gamma, 1e-6, False)
    dx, dg, dx16 = native().rmsnorm_bwd(dy, x, gamma, rstd, dres, True, True)
    xr = x.clone().requires_grad_(True)
    gr = gamma.clone().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * gr
    (yr * dy.float()).sum().backward()
    assert rel(dx, xr.grad + dres) < 1e-4
    assert rel(dg, gr.grad) < 1e-4
    assert rel(dx16.float(), dx) < 1e-2


@pytest.mark.parametrize("mode", [1, 2])
def test_gemm_scatter_epilogue(mode):
    """The scatter epilogue (the fused Newton-Schulz product + all-to-all of
    sharded Muon) on one GPU: destinations are blocks of one local buffer;
    every row (mode 1) or column (mode 2) block lands where its owner reads
    it, bit-identical to the plain GEMM with the same alpha / beta epilogue."""
    from vagus_b200.ops import native
    nb, M, K, N, world = 3, 256, 192, 512, 4
    A = torch.randn(nb, M, M, device=DEV).bfloat16()
    X = torch.randn(nb, M, N, device=DEV).bfloat16()
    ref = torch.empty(nb, M, N, device=DEV, dtype=torch.bfloat16)
    _g(A, False, X, True, ref, X, 1.0, 0.5, False, 1, 0)          # B X + 0.5 X
    span = (M if mode == 1 else N) // world
    if mode == 1:
        recv = torch.zeros(world, nb + 2, span, N, device=DEV, dtype=torch.bfloat16)
        ld, stride = N, span * N
    else:
        recv = torch.zeros(world, nb + 2, M, span, device=DEV, dtype=torch.bfloat16)
        ld, stride = span, M * span
    dst = [recv[o].data_ptr() for o in range(world)]
    rc = native().gemm_scatter(A, False, X, True, X, 1.0, 0.5, dst, mode, span, ld, stride, 2)
    assert rc == 0, rc
    torch.cuda.synchronize()
    for o in range(world):
        got = recv[o, 2:2 + nb]
        want = ref[:, o * span:(o + 1) * span] if mode == 1 else ref[:, :, o * span:(o + 1) * span]
        assert torch.equal(got, want), (mode, o)
        assert recv[o, :2].abs().sum() == 0                           # batch offset respected


def test_bounded_wait_timeout_reports_and_context_survives():
    """Failure detection on the device without a fault: the cross-GPU epoch
    barrier waits for a peer flag that nothing sets (a second heap in this
    process stands in for a peer that never arrives), gives up after its
    budget (set to 1 s here), records kErrTimeoutPeer in the host-mapped error
    word and returns; the host raises on it, and the context keeps working.
    A second barrier issued after the failure returns at once: the error word
    ends every later cross-GPU wait."""
    import time
    from vagus_b200 import ops
    C = ops.native()
    h0, _ = C.comm_heap_create(4096)
    h1, _ = C.comm_heap_create(4096)
    old = C.comm_wait_budget()
    C.comm_set_wait_budget(1.0)
    try:
        t0 = time.time()
        C.comm_barrier([h0, h1], 0, 1)
        torch.cuda.synchronize()
        waited = time.time() - t0
        C.comm_set_wait_budget(30.0)
        t1 = time.time()
        C.comm_barrier([h0, h1], 0, 2)          # the flag never arrives either; the error word ends it
        torch.cuda.synchronize()
        second = time.time() - t1
    finally:
        C.comm_set_wait_budget(old)
    assert C.error_word() == 4, C.error_word()          # kErrTimeoutPeer
    assert 0.5 < waited < 20, waited
    assert second < 5, second
    with pytest.raises(RuntimeError):
        ops.check_error()
    assert C.error_word() == 0
    a = torch.randn(256, 256, device=DEV)
    assert torch.allclose(a @ a, (a.double() @ a.double()).float(), rtol=1e-3, atol=1e-3)
    C.comm_heap_close(h0, True)
    C.comm_heap_close(h1, True)


@pytest.mark.parametrize("b,L,rest", [(2, 1000, (3,)), (3, 257, (4, 37)), (1, 4096, (2, 128)), (2, 5, (1,))])
def test_mobius_scan_kernel_fwd_bwd(b, L, rest):
    """Segmented Mobius scan kernel against the token recurrence in fp64,
    values and gradients (coefficients shaped like the Kalman precision map)."""
    from vagus_b200 import ops
    from vagus_b200.models.kalman import mobius_scan
    g = torch.Generator(device="cuda").manual_seed(0)
    shp = (b, L, *rest)
    m = 2.0 * torch.rand(shp, device="cuda", generator=g)
    w = 0.05 + torch.rand(shp, device="cuda", generator=g)
    a = 0.5 + 0.5 * torch.rand(shp, device="cuda", generator=g)
    coeffs = [1.0 + m * w, m * a, w, a]
    x0 = 0.5 + torch.rand((b, *rest), device="cuda", generator=g)
    leaves = [t.clone().requires_grad_(True) for t in coeffs + [x0]]
    got = ops.mobius_scan(*leaves)
    ref_leaves = [t.double().clone().requires_grad_(True) for t in coeffs + [x0]]
    want = mobius_scan(*ref_leaves, impl="recurrent")
    assert rel(got.double(), want) < 1e-5
    gO = torch.randn(shp, device="cuda", generator=g)
    gg = torch.autograd.grad(got, leaves, gO)
    gw = torch.autograd.grad(want, ref_leaves, gO.double())
    for x, y in zip(gg, gw):
        assert rel(x.double(), y) < 1e-4
    # the model path dispatches to the kernel for CUDA fp32
    assert rel(mobius_scan(*coeffs, x0).double(), want.detach()) < 1e-5


@pytest.mark.parametrize("kalman", ["iso", "diag"])
def test_kalman_layer_kernels_match_torch_path(kalman):
    """A Kalman-delta layer in bf16 on the kernels (Mobius scan kernel, the
    recurrence kernels; the diagonal gain's asymmetric write included) vs the
    same weights on the fp32 torch path, outputs and input gradients."""
    from vagus_b200.models.kalman import KalmanDeltaNet
    torch.manual_seed(0)
    ref = KalmanDeltaNet(256, 2, 128, 128, kalman=kalman, gate_rank=16, impl="torch").to(DEV)
    with torch.no_grad():
        for name, p in ref.named_parameters():
            if name.startswith("womega2"):
                p.normal_(0, 0.05)
    cu = KalmanDeltaNet(256, 2, 128, 128, kalman=kalman, gate_rank=16).to(DEV)
    cu.load_state_dict(ref.state_dict())
    cu = cu.bfloat16()
    x = torch.randn(2, 192, 256, device=DEV)
    xr = x.clone().requires_grad_(True)
    xc = x.bfloat16().requires_grad_(True)
    yr, yc = ref(xr), cu(xc)
    assert rel(yc, yr) < 3e-2, rel(yc, yr)
    dy = torch.randn_like(yr)
    (yr * dy).sum().backward()
    (yc.float() * dy).sum().backward()
    assert rel(xc.grad, xr.grad) < 6e-2, rel(xc.grad, xr.grad)


@pytest.mark.parametrize("rows,owners,N,M,K,a_mn,c32", [(520, 8, 4160, 512, 1024, False, False),
                                                       (512, 2, 1000, 256, 512, False, True),
                                                       (136, 4, 544, 384, 256, True, False),
                                                       (256, 3, 700, 128, 192, False, False)])
def test_gemm_gathered_b(rows, owners, N, M, K, a_mn, c32):
    """GEMM whose B rows come from several owners' buffers (the row shards of
    a weight; here separate local allocations stand in for the peers), tiles
    that straddle an owner boundary included, against the product with the
    concatenated weight."""
    from vagus_b200.ops import native
    W = torch.randn(owners * rows, K, device=DEV).bfloat16()
    shards = [W[o * rows:(o + 1) * rows].clone() for o in range(owners)]
    A = torch.randn(K, M, device=DEV).bfloat16() if a_mn else torch.randn(M, K, device=DEV).bfloat16()
    C = torch.empty(M, N, device=DEV, dtype=torch.float32 if c32 else torch.bfloat16)
    rc = native().gemm_gather(A, a_mn, [s.data_ptr() for s in shards], rows, K, C)
    assert rc == 0, rc
    ref = (A.float().T if a_mn else A.float()) @ W[:N].float().T
    assert rel(C, ref) < 1e-2, rel(C, ref)
