"""Where the time goes: each variant of a ``compare``-style harness under
torch.profiler, with a Chrome trace per variant (chrome://tracing or
ui.perfetto.dev), the top ops, and -- on CUDA -- device time split by kernel
family and by origin (this framework's sm_100a kernels, which live in the
``vagus`` C++ namespace, against library kernels: cuBLAS, NCCL, PyTorch's
own), which is the split that shows whether a hot path fell back to a
library.

Parity: reference ``infra/meter/profiling.py`` (``profile_variants``: every
variant profiled over the shared inputs, top ops printed, one trace each).
"""

from __future__ import annotations

import pathlib
import re
from typing import Callable, Optional

from torch.profiler import ProfilerActivity, profile

from .core import format_table, synchronize, timing_device

# kernel-name families, first match wins
FAMILIES = [
    ("gemm", r"gemm|gemv|cutlass|sm100_xmma|nvjet"),
    ("attention", r"attn|flash|fmha|sdpa"),
    ("delta-rule", r"gdr|kda|intra|scan|mobius"),
    ("conv", r"conv"),
    ("cross-entropy", r"softmax_ce|cross_entropy|\bce_"),
    ("optimizer", r"adamw|muon|newton|foreach|lerp"),
    ("collectives", r"nccl|gather_k|reduce_scatter|barrier_k|comm_|reduce_k|stage_k"),
    ("norms / pointwise", r"norm|swiglu|silu|rope|gate|elementwise|vectorized|copy|fill|cast|mul|add"),
]


def family(kernel: str) -> str:
    low = kernel.lower()
    for fam, pat in FAMILIES:
        if re.search(pat, low):
            return fam
    return "other"


def is_own_kernel(kernel: str) -> bool:
    """True for a kernel of this framework's extension (namespace ``vagus``)."""
    return "vagus::" in kernel


def device_split(prof, steps: int = 1) -> dict:
    """Device ms per step by family, by origin and by kernel from a finished
    profile."""
    fams: dict[str, float] = {}
    origin = {"own": 0.0, "library": 0.0}
    kernels: dict[str, list] = {}
    for ev in prof.key_averages():
        us = getattr(ev, "self_device_time_total", 0.0) or getattr(ev, "self_cuda_time_total", 0.0)
        if us <= 0 or getattr(ev, "device_type", None) is not None and "CUDA" not in str(ev.device_type):
            continue
        ms = us / 1e3 / max(1, steps)
        fams[family(ev.key)] = fams.get(family(ev.key), 0.0) + ms
        origin["own" if is_own_kernel(ev.key) else "library"] += ms
        k = kernels.setdefault(ev.key, [0.0, 0])
        k[0] += ms
        k[1] += ev.count // max(1, steps)
    return {"families_ms": fams, "origin_ms": origin, "kernels": kernels}


def _short(kernel: str, width: int = 90) -> str:
    name = kernel.replace("(anonymous namespace)::", "")
    name = re.sub(r"^void |\(.*$", "", name)
    return name if len(name) <= width else name[:width - 3] + "..."


def render_split(split: dict, top: int = 25) -> str:
    fams, origin = split["families_ms"], split["origin_ms"]
    total = sum(fams.values()) or 1.0
    rows = [[f, f"{ms:.2f}", f"{100 * ms / total:.1f} %"] for f, ms in sorted(fams.items(), key=lambda kv: -kv[1])]
    rows += [[f"[{k} kernels]", f"{v:.2f}", f"{100 * v / total:.1f} %"] for k, v in origin.items()]
    text = format_table(["family", "ms / step", "share"], rows)
    kern = sorted(split.get("kernels", {}).items(), key=lambda kv: -kv[1][0])[:top]
    if kern:
        krows = [[_short(k), str(n), f"{ms:.2f}", f"{100 * ms / total:.1f} %"] for k, (ms, n) in kern]
        text += "\n\n" + format_table(["kernel", "calls / step", "ms / step", "share"], krows)
    return text


def profile_variants(variants: dict[str, Callable], args: tuple = (), kwargs: Optional[dict] = None, *,
                     steps: int = 5, warmup: int = 3, out_dir: str = "profile-output",
                     row_limit: int = 12, device=None) -> dict[str, pathlib.Path]:
    """Profile each variant ``steps`` times after ``warmup`` calls; returns
    ``{name: trace path}`` (a variant that raises is reported and skipped).
    ``device``: where the variants run when no argument tells (closures)."""
    kwargs = kwargs or {}
    device = device if device is not None else timing_device(args, kwargs)
    cuda = device.type == "cuda"
    activities = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if cuda else [])
    out = pathlib.Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    traces: dict[str, pathlib.Path] = {}
    for name, fn in variants.items():
        try:
            for _ in range(warmup):
                fn(*args, **kwargs)
            synchronize(device)
            with profile(activities=activities, record_shapes=True, profile_memory=True) as prof:
                for _ in range(steps):
                    fn(*args, **kwargs)
                synchronize(device)
        except Exception as e:  # noqa: BLE001 -- keep profiling the other variants
            print(f'[meter] profile "{name}" failed: {type(e).__name__}: {e}')
            continue
        path = out / f"{re.sub(r'[^A-Za-z0-9_.-]+', '_', name)}.trace.json"
        prof.export_chrome_trace(str(path))
        traces[name] = path
        key = "self_cuda_time_total" if cuda else "self_cpu_time_total"
        print(f'\n[meter] profile "{name}": {steps} steps on {device}; trace {path}')
        print(prof.key_averages().table(sort_by=key, row_limit=row_limit))
        if cuda:
            print(render_split(device_split(prof, steps)))
    return traces
