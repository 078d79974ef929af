"""Run registry: one JSON record per completed training run.

    python -m vagus_b200.registry RUN_DIR [--out registry] [--incident TEXT ...] [--note TEXT]

The record gathers what a later reader needs to trust and reuse the run:
``run`` (name, directory, code commit, world size, timing), ``recipe`` (the
resolved TrainConfig), ``data`` (store provenance and tokenizer fingerprint
from the run's meta.json), ``results`` (final step and tokens, the mean of
the last five logged losses, median throughput and MFU from metrics.jsonl),
``incidents`` (free text passed on the command line) and ``archive`` (the
checkpoint files with their SHA-256, also written to RUN_DIR/SHA256SUMS).

Parity: reference ``registry/README.md`` and ``registry/*.json`` (one record
per completed run with run / recipe / data / results / incidents / archive).
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

from .data.prepare import sha256_file
from .utils import atomic_write


def _metrics(run_dir: Path) -> list[dict]:
    p = run_dir / "metrics.jsonl"
    if not p.exists():
        return []
    return [json.loads(line) for line in p.read_text().splitlines() if line.strip()]


def build_record(run_dir, incidents=(), note: str | None = None) -> dict:
    run_dir = Path(run_dir)
    meta = json.loads((run_dir / "meta.json").read_text())
    rows = _metrics(run_dir)
    losses = [r["loss"] for r in rows if "loss" in r]
    tput = [r["tokens_per_s"] for r in rows if "tokens_per_s" in r]
    mfu = [r["mfu"] for r in rows if "mfu" in r]
    ckpts = sorted(run_dir.glob("ckpt-*.pt")) + [p for p in (run_dir / "model-final.pt",) if p.exists()]
    archive = [{"file": p.name, "bytes": p.stat().st_size, "sha256": sha256_file(p)} for p in ckpts]
    last = rows[-1] if rows else {}
    return {
        "run": {"name": run_dir.name, "dir": str(run_dir.resolve()), "code": meta.get("code"),
                "created": meta.get("created"), "world_size": meta.get("world_size"), "device": meta.get("device"),
                "torch": meta.get("torch")},
        "recipe": meta.get("config"),
        "data": meta.get("data"),
        "results": {"final_step": last.get("step"), "tokens_seen": last.get("tokens", last.get("tokens_seen")),
                    "loss_tail5": statistics.fmean(losses[-5:]) if losses else None,
                    "tokens_per_s_median": statistics.median(tput) if tput else None,
                    "mfu_median": statistics.median(mfu) if mfu else None,
                    "derived": meta.get("derived")},
        "incidents": list(incidents),
        "note": note,
        "archive": archive,
    }


def write_record(run_dir, out_dir="registry", incidents=(), note: str | None = None) -> Path:
    run_dir = Path(run_dir)
    rec = build_record(run_dir, incidents, note)
    sums = "".join(f'{a["sha256"]}  {a["file"]}\n' for a in rec["archive"])
    atomic_write(run_dir / "SHA256SUMS", lambda f: f.write(sums.encode()))
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    path = out / f"{run_dir.name}.json"
    atomic_write(path, lambda f: f.write(json.dumps(rec, indent=2).encode()))
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description="write the registry record of a completed run")
    ap.add_argument("run_dir")
    ap.add_argument("--out", default="registry")
    ap.add_argument("--incident", action="append", default=[])
    ap.add_argument("--note")
    a = ap.parse_args(argv)
    print(write_record(a.run_dir, a.out, a.incident, a.note))


if __name__ == "__main__":
    main()
