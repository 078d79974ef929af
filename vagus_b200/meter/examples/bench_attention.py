"""Causal attention, forward and forward+backward: this framework's flash
attention (``ops.attention``) against torch SDPA and a materialised-scores
softmax, at a chosen (B, H, L, head dim).

    python -m vagus_b200.meter.examples.bench_attention --B 4 --H 16 --L 4096 --dh 64 128
    python -m vagus_b200.meter.examples.bench_attention --decode --B 8 --prefill 2048 --steps 64

``--decode`` times a whole softmax-attention layer (qk-norm, RoPE, GQA as
given) streaming through its KV cache: a prompt prefill, then single-token
decode steps (lower-right causal attention over the cache).
"""

from __future__ import annotations

import argparse
import faulthandler
import math
import sys

import torch
import torch.nn.functional as F

from ... import ops
from ..compare import compare


def naive(q, k, v):
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    L = q.shape[-2]
    s = s.masked_fill(~torch.ones(L, L, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return (s.softmax(-1) @ v.float()).to(q.dtype)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--dh", type=int, nargs="+", default=[64, 128])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-naive", action="store_true", help="skip the materialised variant (memory)")
    ap.add_argument("--decode", action="store_true", help="streaming prefill / decode of a whole layer")
    ap.add_argument("--prefill", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--kv-heads", type=int, default=None, help="GQA: key/value heads (default: H)")
    ap.add_argument("--variants", nargs="+", default=None, help="subset of ours / sdpa / naive")
    a = ap.parse_args(argv)
    try:
        faulthandler.enable(file=sys.__stderr__)   # a native crash prints every thread's Python stack
    except (AttributeError, OSError, ValueError):  # no real stderr (captured)
        pass
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if a.decode:
        return decode_main(a, dev)
    for dh in a.dh:
        q, k, v = (torch.randn(a.B, a.H, a.L, dh, device=dev, dtype=torch.bfloat16, requires_grad=True)
                   for _ in range(3))
        variants = {"ours": lambda: ops.attention(q, k, v, causal=True),
                    "sdpa": lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True)}
        if not a.no_naive:
            variants["naive"] = lambda: naive(q, k, v)
        if a.variants:
            variants = {n: f for n, f in variants.items() if n in a.variants}
        ref = "sdpa" if "sdpa" in variants else next(iter(variants))
        print(f"\nforward  B={a.B} H={a.H} L={a.L} dh={dh}")
        compare(variants, ref=ref, iters=a.iters, progress=True)
        do = torch.randn_like(q)

        def fb(fn):
            def run():
                out = fn()
                return torch.autograd.grad(out, (q, k, v), do)[0]
            return run
        print(f"forward+backward  B={a.B} H={a.H} L={a.L} dh={dh}")
        compare({n: fb(f) for n, f in variants.items()}, ref=ref, iters=a.iters, progress=True)


def decode_main(a, dev):
    from ...models.attention import SoftmaxAttention
    from ...models.rope import RoPE
    from ._common import decode_bench, render_decode
    dt = torch.bfloat16 if dev == "cuda" else torch.float32
    out = {}
    print(f"streaming layer: B={a.B} H={a.H} kv heads={a.kv_heads or a.H} prefill={a.prefill} decode steps={a.steps}")
    for dh in a.dh:
        dim = a.H * dh
        torch.manual_seed(0)
        rope = RoPE(dim, dh, a.prefill + a.steps).to(dev)
        layer = SoftmaxAttention(dim, a.H, a.kv_heads, 1, None, True, rope=rope).to(dev, dt).eval()
        x = torch.randn(a.B, a.prefill + a.steps, dim, device=dev, dtype=dt)
        out[f"d{dh}"] = r = decode_bench(layer, x, a.prefill, a.steps, iters=a.iters)
        print(render_decode(f"head dim {dh}", r))
    return out


if __name__ == "__main__":
    main()
