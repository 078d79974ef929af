"""Per-rank benchmarking under torchrun, reported the way a data-parallel
job experiences it.

Every rank times the same callable (``core.bench``, CUDA events) after a
barrier; the per-iteration times of all ranks are then gathered as one
(world x iters) tensor on rank 0.  Besides each rank's mean, the report gives
the mean over iterations of the slowest rank's time -- the step time of a job
whose ranks meet at a collective every iteration -- and the slowest / fastest
rank ratio, which separates "every rank is slow" from "one straggler".
Callables that contain collectives make their ranks wait for one another,
which is what the max-over-ranks figure then shows.

Parity: reference ``infra/meter/dist.py`` (``dist_bench``,
``render_dist_table``: barrier-aligned per-rank benches gathered on rank 0
with an imbalance line).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .core import BenchResult, bench, format_table, timing_device


def _barrier(device: torch.device) -> None:
    if device.type == "cuda":
        dist.barrier(device_ids=[device.index or 0])
    else:
        dist.barrier()


def dist_bench(fn: Callable, args: tuple = (), kwargs: Optional[dict] = None, *, name: Optional[str] = None,
               warmup: int = 10, iters: int = 50) -> Optional[dict[int, BenchResult]]:
    """``{rank: BenchResult}`` on rank 0 (each with its per-iteration
    ``samples``), None on the other ranks.  Collective over the default
    group."""
    assert dist.is_initialized(), "init_process_group first"
    rank, world = dist.get_rank(), dist.get_world_size()
    device = timing_device(args, kwargs or {})
    _barrier(device)                     # a late starter must not read as a straggler
    res = bench(fn, args, kwargs, name=name, device=device, warmup=warmup, iters=iters)
    # fixed-size exchange: [failed flag, mean, std, min, max, first, peak, iters samples]
    comm_dev = device if dist.get_backend() == "nccl" else torch.device("cpu")
    row = torch.full((7 + iters,), float("nan"), dtype=torch.float64)
    if not res.failed:
        row[:7] = torch.tensor([0.0, res.mean_ms, res.std_ms, res.min_ms, res.max_ms, res.first_call_ms,
                                float(res.peak_mem if res.peak_mem is not None else -1)], dtype=torch.float64)
        row[7:7 + len(res.samples)] = torch.tensor(res.samples, dtype=torch.float64)
    else:
        row[0] = 1.0
    flat = torch.empty(world * row.numel(), dtype=torch.float64, device=comm_dev)
    dist.all_gather_into_tensor(flat, row.to(comm_dev))
    if rank != 0:
        return None
    table = flat.cpu().view(world, row.numel())
    out: dict[int, BenchResult] = {}
    for r in range(world):
        v = table[r].tolist()
        if v[0] != 0.0:
            out[r] = BenchResult(res.name, f"rank {r}", 0, 0, 0, 0, 0, 0, None, False,
                                 error="failed on that rank" if r != 0 else res.error)
            continue
        peak = None if v[6] < 0 else int(v[6])
        out[r] = BenchResult(res.name, res.device if r == 0 else f"rank {r}", iters, v[1], v[2], v[3], v[4], v[5],
                             peak, res.mem_exact, samples=v[7:7 + iters])
    return out


def job_time(results: dict[int, BenchResult]) -> Optional[float]:
    """Mean over iterations of the slowest rank's time (ms)."""
    ok = [r.samples for r in results.values() if not r.failed and r.samples]
    if len(ok) < 1:
        return None
    n = min(len(s) for s in ok)
    return sum(max(s[i] for s in ok) for i in range(n)) / n


def render_dist_table(results: dict[int, BenchResult]) -> str:
    rows = []
    for r, res in results.items():
        if res.failed:
            rows.append([str(r), f"FAILED: {res.error}"])
            continue
        mem = "n/a" if res.peak_mem is None else f"{res.peak_mem / 2 ** 20:.1f} MiB"
        rows.append([str(r), res.device, f"{res.mean_ms:.3f} ms", f"{res.std_ms:.3f}", f"{res.min_ms:.3f}", mem])
    text = f"[meter] world_size={len(results)}\n" + format_table(["rank", "device", "mean", "std", "min", "peak mem"],
                                                                  rows)
    means = [res.mean_ms for res in results.values() if not res.failed]
    jt = job_time(results)
    if len(means) >= 2 and jt is not None:
        text += (f"\njob step (slowest rank per iteration) {jt:.3f} ms | slowest/fastest rank mean = "
                 f"{max(means) / min(means):.2f}x ({max(means):.3f} / {min(means):.3f} ms)")
    return text
