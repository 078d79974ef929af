"""Where does the time go: each variant under torch.profiler, the top ops
printed and a Chrome trace exported per variant.

Parity: reference ``infra/meter/profiling.py:21-67``.
"""

from __future__ import annotations

import pathlib
from typing import Callable, Optional

from torch.profiler import ProfilerActivity, profile

from ..utils import infer_device
from .core import synchronize


def profile_variants(variants: dict[str, Callable], args: tuple = (), kwargs: Optional[dict] = None, *,
                     steps: int = 5, warmup: int = 3, out_dir: str = "profile-output",
                     row_limit: int = 12) -> dict[str, pathlib.Path]:
    kwargs = kwargs or {}
    device = infer_device(args, kwargs)
    activities = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if device.type == "cuda" else [])
    sort_by = "self_cuda_time_total" if device.type == "cuda" else "self_cpu_time_total"
    out = pathlib.Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    traces = {}
    for name, fn in variants.items():
        try:
            for _ in range(warmup):
                fn(*args, **kwargs)
            synchronize(device)
            with profile(activities=activities, profile_memory=True, record_shapes=True) as prof:
                for _ in range(steps):
                    fn(*args, **kwargs)
                    synchronize(device)
        except Exception as e:
            print(f'[meter] profile "{name}" failed: {type(e).__name__}: {e}')
            continue
        path = out / f"{name}.trace.json"
        prof.export_chrome_trace(str(path))
        traces[name] = path
        print(f'\n[meter] profile "{name}" ({steps} steps on {device}) -- trace: {path}')
        print(prof.key_averages().table(sort_by=sort_by, row_limit=row_limit))
    return traces
