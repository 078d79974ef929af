"""Causal attention, forward and forward+backward: this framework's flash
attention (``ops.attention``) against torch SDPA and a materialised-scores
softmax, at a chosen (B, H, L, head dim).

    python -m vagus_b200.meter.examples.bench_attention --B 4 --H 16 --L 4096 --dh 64 128
"""

from __future__ import annotations

import argparse
import math

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
    a = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    for dh in a.dh:
        q, k, v = (torch.randn(a.B, a.H, a.L, dh, device=dev, dtype=torch.bfloat16, requires_grad=True)
                   for _ in range(3))
        variants = {"ours": lambda: ops.attention(q, k, v, causal=True),
                    "sdpa": lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True)}
        if not a.no_naive:
            variants["naive"] = lambda: naive(q, k, v)
        print(f"\nforward  B={a.B} H={a.H} L={a.L} dh={dh}")
        compare(variants, ref="sdpa", iters=a.iters)
        do = torch.randn_like(q)

        def fb(fn):
            def run():
                out = fn()
                return torch.autograd.grad(out, (q, k, v), do)[0]
            return run
        print(f"forward+backward  B={a.B} H={a.H} L={a.L} dh={dh}")
        compare({n: fb(f) for n, f in variants.items()}, ref="sdpa", iters=a.iters)


if __name__ == "__main__":
    main()
