"""Generic performance meter for callables: timing and peak memory.

CUDA: CUDA-event timing on the launching stream with an L2 flush (a 256 MB
write, larger than the 126 MB L2) before every timed iteration, warm-up first,
and the exact peak-memory delta measured in a separate pass.  CPU: wall clock
around ``fn()`` per iteration and the process RSS delta (approximate).

Parity: reference ``infra/meter/core.py:26-200`` (BenchResult, bench,
synchronize).
"""

from __future__ import annotations

import gc
import resource
import sys
import time
from dataclasses import dataclass
from typing import Callable, Optional

import torch

from ..utils import iter_tensors

L2_FLUSH_BYTES = 256 * 1024 * 1024


@dataclass
class BenchResult:
    name: str
    device: str
    iters: int
    mean_ms: float
    std_ms: float
    min_ms: float
    max_ms: float
    first_call_ms: float
    peak_mem: Optional[int]
    mem_exact: bool
    error: Optional[str] = None
    samples: Optional[list] = None       # per-iteration ms, in order

    @property
    def failed(self) -> bool:
        return self.error is not None



def timing_device(args: tuple = (), kwargs: Optional[dict] = None) -> torch.device:
    """Device whose clock times a call: the first tensor argument's, else the
    current CUDA device when there is one (closures that hold their tensors
    pass no arguments), else the CPU."""
    for t in iter_tensors((args, kwargs or {})):
        return t.device
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")

def synchronize(device: torch.device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def _cuda_times(run, device, iters: int) -> list[float]:
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.int8, device=device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        flush.zero_()
        starts[i].record()
        run()
        ends[i].record()
    torch.cuda.synchronize(device)
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def _cuda_peak(run, device, probes: int = 3) -> int:
    gc.collect()
    torch.cuda.empty_cache()
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    base = torch.cuda.memory_allocated(device)
    for _ in range(probes):
        run()
    torch.cuda.synchronize(device)
    return max(0, torch.cuda.max_memory_allocated(device) - base)


def _rss() -> int:
    factor = 1 if sys.platform == "darwin" else 1024
    return resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * factor


def bench(fn: Callable, args: tuple = (), kwargs: Optional[dict] = None, *, name: Optional[str] = None,
          device: Optional[torch.device] = None, warmup: int = 10, iters: int = 50) -> BenchResult:
    kwargs = kwargs or {}
    device = device or timing_device(args, kwargs)
    label = name or getattr(fn, "__name__", repr(fn))

    def run():
        return fn(*args, **kwargs)

    try:
        gc.collect()
        synchronize(device)
        t0 = time.perf_counter()
        run()
        synchronize(device)
        first = (time.perf_counter() - t0) * 1e3
        for _ in range(max(0, warmup - 1)):
            run()
        synchronize(device)
        if device.type == "cuda":
            times = _cuda_times(run, device, iters)
            peak, exact = _cuda_peak(run, device), True
        else:
            base = _rss()
            times = []
            for _ in range(iters):
                t0 = time.perf_counter()
                run()
                times.append((time.perf_counter() - t0) * 1e3)
            peak, exact = max(0, _rss() - base), False
    except Exception as e:  # a failed variant must not kill the run
        return BenchResult(label, str(device), 0, 0, 0, 0, 0, 0, None, False, error=f"{type(e).__name__}: {e}")
    mean = sum(times) / len(times)
    std = (sum((t - mean) ** 2 for t in times) / len(times)) ** 0.5
    return BenchResult(label, str(device), len(times), mean, std, min(times), max(times), first, peak, exact,
                       samples=list(times))


def format_table(header: list[str], rows: list[list[str]]) -> str:
    """Left-aligned text table with a rule under the header."""
    cells = [list(map(str, header))] + [[str(c) for c in r] for r in rows]
    widths = [max(len(r[i]) if i < len(r) else 0 for r in cells) for i in range(len(header))]
    out = []
    for n, r in enumerate(cells):
        out.append("  ".join(c.ljust(w) for c, w in zip(r, widths)).rstrip())
        if n == 0:
            out.append("  ".join("-" * w for w in widths))
    return "\n".join(out)


def fmt_bytes(nbytes: Optional[int], exact: bool = True) -> str:
    """Human-readable size; ``~`` marks an approximate (RSS-based) figure."""
    if nbytes is None:
        return "n/a"
    units = ["B", "KiB", "MiB", "GiB", "TiB"]
    k = 0
    v = float(nbytes)
    while v >= 1024 and k < len(units) - 1:
        v /= 1024
        k += 1
    return f"{v:.1f} {units[k]}" + ("" if exact else " ~")
