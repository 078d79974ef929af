"""Checkpoint I/O for the two on-disk formats.

* full -- written by the trainer (``ckpt-STEP.pt``, ``recent.pt``): model,
  optimizer, loader and RNG state, resolved config.  Resume material.
* slim -- ``model-final.pt``: ``SLIM_KEYS`` only.  Inference material.

Both carry ``model_name`` / ``model_args`` / ``model`` (FQN-keyed fp32 state
dict), so ``load_model`` accepts either.

Parity: reference ``infra/models/io.py:23-93`` (same keys, same layout).
"""

from __future__ import annotations

from pathlib import Path

import torch
from torch import nn

from ..utils import atomic_write

SLIM_KEYS = ("model_name", "model_args", "tokenizer", "model", "step", "tokens_seen")
_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _as_dtype(dtype):
    if dtype is None or isinstance(dtype, torch.dtype):
        return dtype
    return _DTYPES[dtype]


def is_full_checkpoint(state: dict) -> bool:
    return "optimizer" in state


def load_checkpoint(path, map_location="cpu") -> dict:
    """The raw dict of either format (``weights_only=False``: the full format
    carries numpy RNG state and the loader state)."""
    return torch.load(path, map_location=map_location, weights_only=False)


def load_model(path, device="cpu", dtype=None) -> tuple[nn.Module, dict]:
    """Rebuild the model from a full or slim checkpoint; returns (model, meta)
    with the model in eval mode."""
    from . import build_model
    state = load_checkpoint(path)
    model = build_model(state["model_name"], state["model_args"])
    model.load_state_dict(state["model"])
    dt = _as_dtype(dtype)
    model = model.to(device=device, dtype=dt) if dt is not None else model.to(device)
    model.eval()
    meta = {"model_name": state["model_name"], "model_args": state["model_args"],
            "tokenizer": state.get("tokenizer"), "step": state.get("step"),
            "tokens_seen": state.get("tokens_seen"),
            "format": "full" if is_full_checkpoint(state) else "slim"}
    return model, meta


def slim_state(state: dict, dtype=None) -> dict:
    dt = _as_dtype(dtype)
    weights = {k: (v.to(dt) if dt is not None and v.is_floating_point() else v) for k, v in state["model"].items()}
    out = {k: state[k] for k in SLIM_KEYS if k in state and k != "model"}
    out["model"] = weights
    return out


def export_slim(src, dst, dtype=None) -> Path:
    state = load_checkpoint(src)
    dst = Path(dst)
    atomic_write(dst, lambda f: torch.save(slim_state(state, dtype), f))
    return dst
