"""Microbenchmarks of the native kernels on the shapes of the 340M GDN layer.

    python -m vagus_b200.meter.kernels [case ...] [--B 8] [--L 4096] [--iters 20] [--warmup 5]

Every case is timed with CUDA events after warm-up, with a 256 MB L2 flush
before each timed iteration (``meter.core.bench``), and printed as one line:
time, the algorithmic bytes or FLOPs of one launch, and the fraction of the
measured peak (``MEASURED_PEAKS.json`` at the repository root: STREAM-style
copy bandwidth and the cuBLAS bf16 GEMM rate).  Inputs are random; the
shapes are those of one micro-batch of the 340M GDN model (dim 1024, 4 heads
of 256, conv 4, packed projection width 4160) unless overridden.  Cases:
conv_fwd, conv_bwd (and conv_fwd_h128 / conv_bwd_h128: heads of 128), gates, gdr_intra_fwd, gdr_fwd (intra + recurrence),
gdr_bwd, gdr_rec_fwd, gdr_rec_bwd, gdr_intra_bwd, attn_fwd_d64 / d128,
sdpa_fwd_d64 / d128 (torch's library kernel, for comparison), attn_bwd_d64 / d128, sdpa_bwd_d64 / d128, kda_gated_fwd, kda_gated_bwd, kda_intra_fwd, kda_intra_bwd, kda_gates_fwd / bwd, gemm_fwd, gemm_dgrad, gemm_wgrad, cublas_fwd / dgrad / wgrad (the same shapes on cuBLAS), rmsnorm, rope_fwd / bwd.  With no
case names every
case runs.

Used for the committed ncu summaries: run one case with few iterations under
``ncu -k regex:<kernel> -c 1``.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from .core import bench

ROOT = Path(__file__).resolve().parents[2]


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"], "src": "of measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "src": "of fallback"}


def _cases(B: int, L: int):
    from ..ops import native
    C = native()
    dev = torch.device("cuda")
    D, hd, H = 1024, 256, 4
    T = B * L
    NP = 4 * D + 2 * H + 56          # packed q,k,v,g + a,b, padded to a multiple of 64
    bf = torch.bfloat16
    r = lambda *s, dt=bf: torch.randn(*s, device=dev).to(dt)   # noqa: E731
    cases = {}

    P = r(B, L, NP)
    x = P[:, :, :D]
    w = 0.3 * torch.randn(D, 1, 4, device=dev)
    y, rn = C.conv_silu_fwd(x, w, hd, True)
    dy = r(B, L, D)
    dP = torch.empty_like(P)
    dw = torch.zeros(D * 4, device=dev)
    mb = T * D * 2
    cases["conv_fwd"] = (lambda: C.conv_silu_fwd(x, w, hd, True), 2 * mb, None)
    cases["conv_bwd"] = (lambda: C.conv_silu_bwd(dy, x, w, rn, dP[:, :, :D], dw, hd, True), 3 * mb, None)
    # the same stream split into heads of 128 (the per-channel-gate layers' q / k)
    y1, rn1 = C.conv_silu_fwd(x, w, 128, True)
    cases["conv_fwd_h128"] = (lambda: C.conv_silu_fwd(x, w, 128, True), 2 * mb, None)
    cases["conv_bwd_h128"] = (lambda: C.conv_silu_bwd(dy, x, w, rn1, dP[:, :, :D], dw, 128, True), 3 * mb, None)

    ab = P.reshape(T, NP)[:, 4 * D:4 * D + 2 * H]
    A_log, dt_bias = torch.randn(H, device=dev), torch.randn(H, device=dev)
    cases["gates"] = (lambda: C.gdn_gates_fwd(ab, A_log, dt_bias, H), T * 2 * H * (2 + 8), None)

    BH = B * H
    from ..ops.gdn import _gdr_fwd, _gdr_bwd
    q = torch.nn.functional.normalize(torch.randn(B, L, H, hd, device=dev), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(B, L, H, hd, device=dev), dim=-1).to(bf)
    v = r(B, L, H, hd)
    g = -torch.rand(B, L, H, device=dev) * 0.1
    beta = torch.rand(B, L, H, device=dev)
    scale = hd ** -0.5
    nc = L // 64
    # per chunk: K K^T, Q K^T, W = T(bGK), U = T(bV): 4 x 2*64*64*256; inverse ~64^3/3
    intra = BH * nc * (4 * 2 * 64 * 64 * hd + 2 * 64 ** 3 // 3)
    # per chunk: W S, Qh S, Kt^T V': 3 x 2*64*256*256, plus A V' (2*64*64*256)
    rec = BH * nc * (3 * 2 * 64 * hd * hd + 2 * 64 * 64 * hd)
    cases["gdr_intra_fwd"] = (lambda: C.gdr_intra_fwd(q, k, v, g, beta, scale), None, intra)
    cases["gdr_fwd"] = (lambda: _gdr_fwd(q, k, v, g, beta, None, scale), None, intra + rec)
    o, _, saved = _gdr_fwd(q, k, v, g, beta, None, scale)
    do = torch.randn_like(o)
    cases["gdr_bwd"] = (lambda: _gdr_bwd(saved, do, None, scale, False), None, 2 * (intra + rec))
    # the two stages separately (inputs from one forward)
    W_, Qh, Kt, A_, U_, gC = C.gdr_intra_fwd(q, k, v, g, beta, scale)
    cases["gdr_rec_fwd"] = (lambda: C.gdr_rec_fwd(W_, Qh, Kt, A_, U_, gC, None, True, H), None, rec)
    _, Vp, states, _ = C.gdr_rec_fwd(W_, Qh, Kt, A_, U_, gC, None, True, H)
    dO = torch.randn(B, L, H, hd, device=dev).to(bf)
    cases["gdr_rec_bwd"] = (lambda: C.gdr_rec_bwd(W_, Qh, Kt, A_, Vp, gC, states, dO, None, False), None, 2 * rec)
    rb = C.gdr_rec_bwd(W_, Qh, Kt, A_, Vp, gC, states, dO, None, False)
    cases["gdr_intra_bwd"] = (lambda: C.gdr_intra_bwd(q, k, v, g, beta, *rb[:6], scale), None, 2 * intra)

    # KDA gated intra-chunk products at the 340M KDA shape (4 heads, dk 128)
    dkk = 128
    Nq = B * 4 * (L // 64)
    Qg = torch.randn(Nq, 64, dkk, device=dev)
    Kg = torch.randn(Nq, 64, dkk, device=dev)
    Gg = (-torch.rand(Nq, 64, dkk, device=dev) * 0.05).cumsum(1)
    dA1, dA2 = torch.randn(Nq, 64, 64, device=dev), torch.randn(Nq, 64, 64, device=dev)
    kfl = Nq * 64 * 65 // 2 * dkk * 4                 # pairs x channels x (exp-weighted FMAs)
    cases["kda_gated_fwd"] = (lambda: C.kda_gated_fwd(Qg, Kg, Gg), None, kfl)
    cases["kda_gated_bwd"] = (lambda: C.kda_gated_bwd(Qg, Kg, Gg, dA1, dA2), None, 2 * kfl)
    # the fused KDA intra stage (kda_intra.cu) at the same shape, value head dim 256
    qa = torch.nn.functional.normalize(torch.randn(B, L, 4, dkk, device=dev), dim=-1).to(bf)
    ka = torch.nn.functional.normalize(torch.randn(B, L, 4, dkk, device=dev), dim=-1).to(bf)
    va = r(B, L, 4, 256)
    ga = -torch.rand(B, L, 4, dkk, device=dev) * 0.05
    ba = torch.rand(B, L, 4, device=dev)
    kda_in = (qa, ka, va, ga, ba, dkk ** -0.5)
    # per chunk: two gated products (64 x 64 x 128), W = T(bGK), U = T(bV), the 64 x 64 inverse
    kintra = Nq * (2 * 2 * 64 * 64 * dkk + 2 * 64 * 64 * (dkk + 256) + 2 * 64 ** 3 // 3)
    cases["kda_intra_fwd"] = (lambda: C.kda_intra_fwd(*kda_in), None, kintra)
    # the per-channel gate from the low-rank projection (4 heads x 128 channels) and its backward
    fg = r(B * L, 4 * dkk)
    bg = r(B * L, 4)
    A_lg, dtb = torch.randn(4, device=dev) * 0.1, torch.randn(4 * dkk, device=dev) * 0.1
    cases["kda_gates_fwd"] = (lambda: C.kda_gates_fwd(fg, bg, A_lg, dtb, 4, dkk), B * L * 4 * dkk * (2 + 4), None)
    dgg, dbg = torch.randn(B * L, 4 * dkk, device=dev), torch.randn(B * L, 4, device=dev)
    dfg, dbb = torch.empty_like(fg), torch.empty_like(bg)
    cases["kda_gates_bwd"] = (lambda: C.kda_gates_bwd(dgg, dbg, fg, bg, A_lg, dtb, dfg, dbb, 4, dkk),
                              B * L * 4 * dkk * (4 + 2 + 2), None)
    kout = C.kda_intra_fwd(*kda_in)
    kgr = [torch.randn_like(t).to(t.dtype) for t in kout]
    cases["kda_intra_bwd"] = (lambda: C.kda_intra_bwd(*kda_in[:5], kgr[0], kgr[1], kgr[2], kgr[3].float(), kgr[4],
                                                      kgr[5], kda_in[5]), None, 2 * kintra)

    # Kalman precision recurrence (Mobius scan) at the diagonal KDN shape: 4 heads x 128 channels
    from ..models.kalman import mobius_scan as _mob
    Rm = 4 * 128
    cm = [0.05 + torch.rand(B, L, Rm, device=dev) for _ in range(4)]
    x0m = torch.rand(B, Rm, device=dev) + 0.5
    mbytes = 5 * B * L * Rm * 4                        # four inputs read (twice: compose, replay) + x written
    cases["mobius_fwd"] = (lambda: C.mobius_fwd(*cm, x0m), mbytes + 4 * B * L * Rm * 4, None)
    xm = C.mobius_fwd(*cm, x0m)
    gm = torch.randn_like(xm)
    cases["mobius_bwd"] = (lambda: C.mobius_bwd(*cm, x0m, xm, gm), 15 * B * L * Rm * 4, None)
    cases["mobius_torch"] = (lambda: _mob(*cm, x0m, impl="torch"), mbytes, None)

    from ..ops._core import gemm
    a = r(T, D)
    wpk = r(NP, D)
    c = torch.empty(T, NP, device=dev, dtype=bf)
    gp = r(T, NP)
    da = torch.empty(T, D, device=dev, dtype=bf)
    dwp = torch.zeros(NP, D, device=dev)
    fl = 2 * T * D * NP
    cases["gemm_fwd"] = (lambda: gemm(a, False, wpk, False, c), None, fl)            # x W^T
    # the same product with W's rows gathered from 8 owners' buffers (the fused
    # all-gather's GEMM; local buffers stand in for the peers): 520-row shards,
    # so tiles that straddle an owner boundary take 8-row boxes
    owners = 8
    rows_o = ((NP + owners - 1) // owners + 7) // 8 * 8      # rows per owner, a multiple of 8
    shards = [r(rows_o, D) for _ in range(owners)]
    ptrs = [t.data_ptr() for t in shards]
    cases["gemm_gather_fwd"] = (lambda: C.gemm_gather(a, False, ptrs, rows_o, D, c), None, fl)
    cases["gemm_dgrad"] = (lambda: gemm(gp, False, wpk, True, da), None, fl)         # dy W
    cases["gemm_wgrad"] = (lambda: gemm(gp, True, a, True, dwp, atomic=True), None, fl)  # dW += dy^T x
    # cuBLAS (torch.matmul) on the same three products, for the comparison on
    # the same shape; the wgrad one writes a fresh fp32 product (no accumulate)
    cases["cublas_fwd"] = (lambda: torch.matmul(a, wpk.t()), None, fl)
    cases["cublas_dgrad"] = (lambda: torch.matmul(gp, wpk), None, fl)
    cases["cublas_wgrad"] = (lambda: torch.matmul(gp.t(), a), None, fl)

    # causal attention at the Transformer++ 340M shape (16 heads of 64) and
    # the hybrid 1.3B softmax layers (16 heads of 128)
    import math as _m
    from torch.nn import functional as F
    for hd_a, Ha in ((64, 16), (128, 16)):
        qa = r(B, Ha, L, hd_a)
        ka = r(B, Ha, L, hd_a)
        va = r(B, Ha, L, hd_a)
        fl_a = 2 * 2 * B * Ha * L * L * hd_a / 2                       # causal half of QK^T and PV
        sc = 1.0 / _m.sqrt(hd_a)
        cases[f"attn_fwd_d{hd_a}"] = (lambda qa=qa, ka=ka, va=va, sc=sc: C.attn_fwd(qa, ka, va, True, sc), None, fl_a)
        cases[f"sdpa_fwd_d{hd_a}"] = (lambda qa=qa, ka=ka, va=va: F.scaled_dot_product_attention(qa, ka, va, is_causal=True),
                                      None, fl_a)
        oa, lsea = C.attn_fwd(qa, ka, va, True, sc)
        doa = torch.randn_like(oa)
        cases[f"attn_bwd_d{hd_a}"] = (lambda qa=qa, ka=ka, va=va, oa=oa, lsea=lsea, doa=doa, sc=sc:
                                      C.attn_bwd(qa, ka, va, oa, lsea, doa, True, sc), None, 2.5 * fl_a)
        qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (qa, ka, va))
        og = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
        cases[f"sdpa_bwd_d{hd_a}"] = (lambda og=og, doa=doa, ins=(qg, kg, vg):
                                      torch.autograd.grad(og, ins, doa, retain_graph=True), None, 2.5 * fl_a)

    xs = r(T, D)
    gamma = torch.ones(D, device=dev)
    cases["rmsnorm"] = (lambda: C.rmsnorm_fwd(xs, gamma, 1e-6, False), 2 * T * D * 2, None)
    # qk-norm + RoPE at the Transformer++ shape (16 heads x 64)
    xr4 = r(B, L, 16, 64)
    gr4 = torch.ones(64, device=dev)
    cs = torch.randn(L, 32, device=dev)
    sn = torch.randn(L, 32, device=dev)
    cases["rope_fwd"] = (lambda: C.qk_norm_rope_fwd(xr4, gr4, cs, sn, 1e-6), 2 * xr4.numel() * 2, None)
    y4, rs4 = C.qk_norm_rope_fwd(xr4, gr4, cs, sn, 1e-6)
    dy4 = torch.randn_like(y4)
    cases["rope_bwd"] = (lambda: C.qk_norm_rope_bwd(dy4, xr4, gr4, cs, sn, rs4), 3 * xr4.numel() * 2, None)
    return cases


def _spin(ms: float) -> None:
    import time
    x = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while (time.perf_counter() - t0) * 1e3 < ms:
        for _ in range(8):
            x @ x
        torch.cuda.synchronize()
    del x


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("case", nargs="*")
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--spin-ms", type=float, default=1000.0,
                    help="bf16 matmuls before the first case, so it is not timed while the clocks ramp up")
    a = ap.parse_args(argv)
    peaks = _peaks()
    cases = _cases(a.B, a.L)
    names = a.case or list(cases)
    _spin(a.spin_ms)
    for n in names:
        fn, nbytes, flops = cases[n]
        res = bench(fn, name=n, device=torch.device("cuda"), warmup=a.warmup, iters=a.iters)
        us = res.mean_ms * 1e3
        if nbytes:
            gbs = nbytes / us / 1e3
            print(f"{n:14s} {us:9.1f} us (min {res.min_ms * 1e3:8.1f})  {gbs:7.0f} GB/s  "
                  f"{gbs / peaks['hbm_gbs']:.2f} {peaks['src']} HBM")
        else:
            tf = flops / us / 1e6
            print(f"{n:14s} {us:9.1f} us (min {res.min_ms * 1e3:8.1f})  {tf:7.0f} TF/s  "
                  f"{tf / peaks['tflops']:.2f} {peaks['src']} bf16")


if __name__ == "__main__":
    main()
