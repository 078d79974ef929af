"""The chunked delta-rule family, forward and forward+backward: the sm_100a
kernels (``ops.gdr_chunk`` for the scalar gate, ``ops.kda_chunk`` for the
per-channel gate / gated linear attention / DeltaNet) against the torch
chunk oracle (``models.scans.chunk_scan``, fp32).

    python -m vagus_b200.meter.examples.bench_linear_attention --B 4 --L 4096 --H 16 --dk 128 --dv 128
    python -m vagus_b200.meter.examples.bench_linear_attention --decode --B 8 --prefill 2048 --steps 64

``--decode`` times a whole GatedDeltaNet layer streaming through its cache
(prefill of a prompt, then single-token decode steps on the decode kernel)
for each mode, against the same layer on the torch path.

Parity: reference ``infra/meter/examples/bench_linear_attention.py`` and
``bench_kda_kernel.py`` (there: fla's Triton kernels against a torch scan).
"""

from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F

from ... import ops
from ...models.scans import chunk_scan
from ..compare import compare


def inputs(B, L, H, dk, dv, gate: str, device):
    q = F.normalize(torch.randn(B, L, H, dk, device=device), dim=-1).bfloat16()
    k = F.normalize(torch.randn(B, L, H, dk, device=device), dim=-1).bfloat16()
    v = torch.randn(B, L, H, dv, device=device).bfloat16()
    beta = torch.rand(B, L, H, device=device)
    if gate == "scalar":
        g = -0.1 * torch.rand(B, L, H, device=device)
    elif gate == "vector":
        g = -0.1 * torch.rand(B, L, H, dk, device=device)
    else:
        g = None
    return q, k, v, g, beta


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--dk", type=int, default=128)
    ap.add_argument("--dv", type=int, default=128)
    ap.add_argument("--modes", nargs="+", default=["gdn", "kda", "gla", "deltanet"],
                    help="gdn (scalar gate), kda (per-channel), gla (no delta rule), deltanet (no gate)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no-oracle", action="store_true", help="skip the torch scan (slow at large L)")
    ap.add_argument("--decode", action="store_true", help="streaming prefill / decode of a whole layer")
    ap.add_argument("--prefill", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=64)
    a = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if a.decode:
        return decode_main(a, dev)
    scale = a.dk ** -0.5
    for mode in a.modes:
        gate = {"gdn": "scalar", "kda": "vector", "gla": "vector", "deltanet": "none"}[mode]
        delta = mode != "gla"
        q, k, v, g, beta = inputs(a.B, a.L, a.H, a.dk, a.dv, gate, dev)
        leaves = [t.requires_grad_(True) for t in (q, k, v)]
        if mode == "gdn" and dev == "cuda":
            kern = lambda: ops.gdr_chunk(q, k, v, g, beta, None, scale=scale)[0]          # noqa: E731
        else:
            kern = lambda: ops.kda_chunk(q, k, v, g, beta, None, scale=scale, delta=delta)[0]   # noqa: E731
        variants = {}
        if not a.no_oracle:
            variants["torch"] = lambda: chunk_scan(q.float(), k.float(), v.float(), g, beta, None, scale=scale,
                                                   delta=delta)[0]
        if dev == "cuda":
            variants["ours"] = kern
        do = torch.randn(a.B, a.L, a.H, a.dv, device=dev)

        def fb(fn):
            def run():
                out = fn()
                return torch.autograd.grad(out, leaves, do.to(out.dtype))[0]
            return run
        ref = "torch" if "torch" in variants else "ours"
        print(f"\n{mode}: forward  B={a.B} L={a.L} H={a.H} dk={a.dk} dv={a.dv}")
        compare(variants, ref=ref, iters=a.iters)
        print(f"{mode}: forward+backward")
        compare({n: fb(f) for n, f in variants.items()}, ref=ref, iters=a.iters)


def decode_main(a, dev):
    from ...models.gdn import GatedDeltaNet
    from ._common import decode_bench, render_decode
    dim = a.H * a.dv
    dt = torch.bfloat16 if dev == "cuda" else torch.float32
    x = torch.randn(a.B, a.prefill + a.steps, dim, device=dev, dtype=dt)
    print(f"streaming layer: B={a.B} H={a.H} dk={a.dk} dv={a.dv} prefill={a.prefill} decode steps={a.steps}")
    out = {}
    for mode in a.modes:
        gate = {"gdn": "scalar", "kda": "vector", "gla": "vector", "deltanet": "none"}[mode]
        for impl in (("auto", "torch") if dev == "cuda" else ("torch",)):
            torch.manual_seed(0)
            layer = GatedDeltaNet(dim, a.H, a.dk, a.dv, gate=gate, delta=mode != "gla", gate_rank=16,
                                  impl=impl).to(dev, dt).eval()
            r = decode_bench(layer, x, a.prefill, a.steps, iters=a.iters)
            out[f"{mode}/{impl}"] = r
            print(render_decode(f"{mode}/{impl}", r))
    return out


if __name__ == "__main__":
    main()
