"""Small shared helpers: crash-safe writes, code identity, device/dtype inference.

Parity: reference ``infra/utils.py:11-67`` (atomic_write, git_state,
infer_device, infer_dtype).
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path
from typing import Callable, Iterator

import torch
from torch import nn

__all__ = ["atomic_write", "git_state", "infer_device", "infer_dtype", "iter_tensors"]


def atomic_write(path: str | Path, write_fn: Callable) -> None:
    """Write ``path`` through a sibling temp file and ``os.replace``.

    Readers therefore see either no file or a complete one; a crash mid-write
    leaves only the ``.tmp`` sibling behind.  ``write_fn`` receives the open
    binary handle.
    """
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "wb") as fh:
        write_fn(fh)
        fh.flush()
        os.fsync(fh.fileno())
    os.replace(tmp, path)


def git_state() -> dict:
    """``{'commit': sha | None, 'dirty': bool | None}`` of this source tree."""
    root = Path(__file__).resolve().parents[2]

    def run(*args: str) -> str:
        return subprocess.run(["git", *args], cwd=root, capture_output=True,
                              text=True, check=True).stdout.strip()

    try:
        return {"commit": run("rev-parse", "HEAD"), "dirty": bool(run("status", "--porcelain"))}
    except Exception:  # no git, or not a checkout
        return {"commit": None, "dirty": None}


def iter_tensors(obj) -> Iterator[torch.Tensor]:
    if isinstance(obj, torch.Tensor):
        yield obj
    elif isinstance(obj, nn.Module):
        yield from obj.parameters()
        yield from obj.buffers()
    elif isinstance(obj, dict):
        for v in obj.values():
            yield from iter_tensors(v)
    elif isinstance(obj, (list, tuple, set)):
        for v in obj:
            yield from iter_tensors(v)


def infer_device(*objs) -> torch.device:
    """Device of the first tensor found in ``objs`` (CPU when there is none)."""
    for t in iter_tensors(objs):
        return t.device
    return torch.device("cpu")


def infer_dtype(*objs) -> torch.dtype:
    """Working dtype: the first floating tensor's dtype; integer tensors only
    count when nothing floating is present."""
    fallback = None
    for t in iter_tensors(objs):
        if t.is_floating_point() or t.is_complex():
            return t.dtype
        if fallback is None:
            fallback = t.dtype
    return fallback if fallback is not None else torch.get_default_dtype()
