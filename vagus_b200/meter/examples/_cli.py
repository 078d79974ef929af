"""Command-line plumbing shared by the checkpoint probes."""

from __future__ import annotations

import argparse
import json

import torch

from ._common import parse_ckpts, windows


def probe_args(doc: str) -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=doc.split("\n")[0])
    ap.add_argument("--ckpt", action="append", required=True, help="NAME=checkpoint path (repeatable)")
    ap.add_argument("--data", required=True, help="tokenized store (a directory with a manifest)")
    ap.add_argument("--context-len", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--batches", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--dtype", default=None, help="load the weights in this dtype (default: as saved)")
    ap.add_argument("--json", default=None, help="write the results here as well")
    return ap


def run_probe(a, probe, render) -> dict:
    from ...models.io import load_model
    batches = windows(a.data, a.context_len, a.batch, a.batches, a.seed)
    results = {}
    for name, path in parse_ckpts(a.ckpt).items():
        model, _ = load_model(path, a.device, a.dtype)
        results[name] = probe(model, [b.to(a.device) for b in batches])
        print(f"== {name} ({path})")
        print(render(results[name]))
        del model
    if a.json:
        with open(a.json, "w") as f:
            json.dump(results, f, indent=1)
    return results
