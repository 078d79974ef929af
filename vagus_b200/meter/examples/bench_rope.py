"""qk RMSNorm + rotary embedding: the fused kernel (``ops.qk_norm_rope``)
against the same arithmetic in plain torch, forward+backward.

    python -m vagus_b200.meter.examples.bench_rope --B 8 --L 4096 --H 16 --dh 64
"""

from __future__ import annotations

import argparse

import torch

from ... import ops
from ...models.rope import RoPE
from ..compare import compare


def torch_ref(x, gamma, tables, eps):
    cos, sin = tables
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * gamma
    pairs = xf.reshape(*xf.shape[:-1], xf.shape[-1] // 2, 2)      # interleaved (even, odd) pairs
    x0, x1 = pairs[..., 0], pairs[..., 1]
    c, s = cos.float()[None, :, None, :], sin.float()[None, :, None, :]
    return torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), -1).reshape(x.shape).to(x.dtype)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--dh", type=int, default=64)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    rope = RoPE(a.dh, a.dh, a.L).to(dev)
    tables = rope.tables(a.L, 0)
    x = torch.randn(a.B, a.L, a.H, a.dh, device=dev, dtype=torch.bfloat16, requires_grad=True)
    gamma = torch.ones(a.dh, device=dev, requires_grad=True)
    dy = torch.randn_like(x)

    def fb(fn):
        def run():
            return torch.autograd.grad(fn(), (x,), dy)[0]
        return run
    compare({"torch": fb(lambda: torch_ref(x, gamma, tables, 1e-6)),
             "ours": fb(lambda: ops.qk_norm_rope(x, gamma, tables, 1e-6))}, ref="torch", iters=a.iters)


if __name__ == "__main__":
    main()
