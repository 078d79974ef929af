"""Barrier-aligned per-rank benchmarking under torchrun; results gathered on
rank 0 with a slowest / fastest rank ratio (straggler report).

Parity: reference ``infra/meter/dist.py:22-77``.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch.distributed as dist

from ..utils import infer_device
from .core import BenchResult, bench


def dist_bench(fn: Callable, args: tuple = (), kwargs: Optional[dict] = None, *, name: Optional[str] = None,
               warmup: int = 10, iters: int = 50) -> Optional[dict[int, BenchResult]]:
    assert dist.is_initialized(), "call torch.distributed.init_process_group first"
    rank, world = dist.get_rank(), dist.get_world_size()
    device = infer_device(args, kwargs or {})
    if device.type == "cuda":
        dist.barrier(device_ids=[device.index or 0])
    else:
        dist.barrier()
    result = bench(fn, args, kwargs, name=name, device=device, warmup=warmup, iters=iters)
    gathered: list = [None] * world
    dist.all_gather_object(gathered, result)
    return {i: r for i, r in enumerate(gathered)} if rank == 0 else None


def render_dist_table(results: dict[int, BenchResult]) -> str:
    ok = {i: r for i, r in results.items() if not r.failed}
    lines = [f"[meter] world_size={len(results)}"]
    header = ["rank", "device", "mean", "std", "min", "peak mem"]
    rows = [header]
    for i, r in results.items():
        if r.failed:
            rows.append([str(i), r.device, f"FAILED: {r.error}", "", "", ""])
            continue
        mem = "n/a" if r.peak_mem is None else f"{r.peak_mem / 2**20:.1f} MiB"
        rows.append([str(i), r.device, f"{r.mean_ms:.3f} ms", f"{r.std_ms:.3f}", f"{r.min_ms:.3f}", mem])
    widths = [max(len(row[c]) for row in rows) for c in range(len(header))]
    for j, row in enumerate(rows):
        lines.append("  ".join(c.ljust(w) for c, w in zip(row, widths)).rstrip())
        if j == 0:
            lines.append("  ".join("-" * w for w in widths))
    if len(ok) >= 2:
        means = [r.mean_ms for r in ok.values()]
        lines.append(f"group mean {sum(means) / len(means):.3f} ms | slowest/fastest rank = "
                     f"{max(means) / min(means):.2f}x ({max(means):.3f} / {min(means):.3f} ms)")
    return "\n".join(lines)
