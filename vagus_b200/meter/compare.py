"""Head-to-head of several implementations of one computation on shared
inputs: each variant is timed by ``core.bench`` (so its cold first call is
measured too), then run once more and its output checked against the
reference variant's.

Outputs may be tensors or nested tuples / lists / dicts of them; agreement is
judged leaf by leaf -- the largest absolute difference and the largest
relative Frobenius error over the leaves -- so a variant returning (out,
state) is compared on both.  A variant that raises is reported, not fatal;
variants must not modify their inputs.

Parity: reference ``infra/meter/compare.py`` (``compare``, ``render_table``:
speed, peak memory and deviation from a reference variant, one row each).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Iterator, Optional

import torch

from .core import BenchResult, bench, fmt_bytes, format_table, timing_device


@dataclass
class Agreement:
    """How closely a variant's output matches the reference's."""
    max_abs: float          # max over leaves of max |a - b|
    max_rel: float          # max over leaves of ||a - b|| / ||b||
    leaves: int


def _leaves(x: Any, path: str = "") -> Iterator[tuple[str, Any]]:
    if isinstance(x, torch.Tensor) or x is None or isinstance(x, (int, float)):
        yield path, x
    elif isinstance(x, dict):
        for k in sorted(x):
            yield from _leaves(x[k], f"{path}.{k}")
    elif isinstance(x, (tuple, list)):
        for i, v in enumerate(x):
            yield from _leaves(v, f"{path}[{i}]")
    else:
        yield path, x


def agreement(out: Any, ref: Any) -> Optional[Agreement]:
    """Leaf-wise agreement of ``out`` with ``ref``; None when the structures
    hold no comparable tensors; an infinite error when they differ in shape
    or structure."""
    a, b = dict(_leaves(out)), dict(_leaves(ref))
    if a.keys() != b.keys():
        return Agreement(float("inf"), float("inf"), 0)
    worst_abs = worst_rel = 0.0
    n = 0
    for k, rv in b.items():
        ov = a[k]
        if not (isinstance(ov, torch.Tensor) and isinstance(rv, torch.Tensor)):
            continue
        if ov.shape != rv.shape:
            return Agreement(float("inf"), float("inf"), n)
        d = (ov.detach().double() - rv.detach().double())
        worst_abs = max(worst_abs, d.abs().max().item() if d.numel() else 0.0)
        denom = rv.detach().double().norm().item()
        worst_rel = max(worst_rel, d.norm().item() / denom if denom > 0 else (0.0 if d.norm() == 0 else float("inf")))
        n += 1
    return Agreement(worst_abs, worst_rel, n) if n else None


def compare(variants: dict[str, Callable], args: tuple = (), kwargs: Optional[dict] = None, *,
            ref: Optional[str] = None, warmup: int = 10, iters: int = 50, check: bool = True,
            verbose: bool = True, device: Optional[torch.device] = None,
            progress: bool = False) -> dict[str, BenchResult]:
    """Time every variant on ``args`` / ``kwargs`` and (``check``) compare
    its output with variant ``ref`` (default: the first).  Returns
    ``{name: BenchResult}``; each result carries ``.vs_ref`` (an
    ``Agreement`` or None).  ``progress`` names each variant (flushed)
    before it runs, so a crash inside one is attributed."""
    kwargs = kwargs or {}
    ref = ref or next(iter(variants))
    device = device or timing_device(args, kwargs)
    results: dict[str, BenchResult] = {}
    outputs: dict[str, Any] = {}
    for name, fn in variants.items():
        if progress:
            print(f"[meter] timing {name}", flush=True)
        r = bench(fn, args, kwargs, name=name, device=device, warmup=warmup, iters=iters)
        r.vs_ref = None
        results[name] = r
        if check and not r.failed:
            try:
                with torch.no_grad():
                    outputs[name] = fn(*args, **kwargs)
            except Exception:  # noqa: BLE001 -- bench() already recorded the failure mode
                outputs[name] = None
    if check and ref in outputs:
        for name, out in outputs.items():
            if name != ref and out is not None:
                results[name].vs_ref = agreement(out, outputs[ref])
    if verbose:
        print(render_table(results, ref=ref))
    return results


def render_table(results: dict[str, BenchResult], *, ref: str) -> str:
    base = results.get(ref)
    rows = []
    for name, r in results.items():
        if r.failed:
            rows.append([name, f"FAILED: {r.error}"])
            continue
        if name == ref:
            speed, dev = "1.00x (ref)", "ref"
        else:
            speed = f"{base.mean_ms / r.mean_ms:.2f}x" if base is not None and not base.failed else "n/a"
            ag = getattr(r, "vs_ref", None)
            dev = "-" if ag is None else f"{ag.max_abs:.2e} / {ag.max_rel:.2e}"
        rows.append([name, f"{r.mean_ms:.3f} ms", f"{r.std_ms:.3f}", f"{r.min_ms:.3f}", speed,
                     f"{r.first_call_ms:.1f} ms", fmt_bytes(r.peak_mem, r.mem_exact), dev])
    dev_name = next(iter(results.values())).device if results else "?"
    header = ["variant", "mean", "std", "min", "speedup", "first call", "peak mem", "max|d| / rel vs ref"]
    return f"[meter] device={dev_name}\n" + format_table(header, rows)
