"""Evaluation entry point: ``vagus-b200-eval recipe.yaml [key=value ...]``.

recipe -> subjects x tasks -> record.  Subject-major: each checkpoint is
loaded once, every task runs on it, then it is freed; pairing happens after
from the stored per-item arrays.  The run directory (config.yaml, meta.json,
results.json written after every task, samples/, log.txt) is never silently
overwritten; a copy of the whole record goes to the registry directory.

Parity: reference ``infra/eval/main.py:34-216``.
"""

from __future__ import annotations

import argparse
import gc
import json
import sys
import time
from dataclasses import asdict, dataclass
from datetime import datetime
from pathlib import Path

import torch
import yaml

from ..config import apply_overrides, load_yaml
from ..inference import Generator
from ..utils import atomic_write, git_state
from .core import EvalCtx, Subject, TaskResult, sha256_file
from .pairs import paired
from .tasks import TASKS

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@dataclass
class EvalConfig:
    eval_name: str
    subjects: list
    tasks: list
    device: str = "auto"
    dtype: str = "bfloat16"
    seed: int = 0
    out_root: str = "runs/eval"
    run_dir: str | None = None
    registry_dir: str | None = "registry/eval"
    n_boot: int = 2000

    @classmethod
    def from_yaml(cls, path, overrides=()) -> "EvalConfig":
        return cls(**apply_overrides(load_yaml(path), overrides))


def resolve_device(name: str) -> torch.device:
    if name != "auto":
        return torch.device(name)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def load_subject(spec, device, dtype) -> Subject:
    spec = {"ckpt": spec} if isinstance(spec, str) else dict(spec)
    src = Path(spec.get("ckpt") or spec["run"])
    ckpt, label = (src / "model-final.pt", src.name) if src.is_dir() else (src, src.stem)
    label = spec.get("label") or label
    gen, meta = Generator.from_checkpoint(ckpt, device=device, dtype=dtype, tokenizer_id=spec.get("tokenizer_id"),
                                         with_meta=True)
    run_meta = None
    beside = Path(spec["run_meta"]) if spec.get("run_meta") else ckpt.parent / "meta.json"
    if beside.exists():
        cand = json.loads(beside.read_text())
        if "config" in cand and "data" in cand:
            run_meta = cand
        elif spec.get("run_meta"):
            raise ValueError(f"{beside} is not a train run meta.json")
    return Subject(label=label, path=ckpt.resolve(), sha256=sha256_file(ckpt), meta=meta, generator=gen,
                   run_meta=run_meta)


def _write_json(path: Path, obj) -> None:
    atomic_write(path, lambda f: f.write(json.dumps(obj, indent=2).encode()))


def evaluate(config: EvalConfig) -> Path:
    code = git_state()
    commit8 = (code["commit"] or "nogit")[:8]
    run_dir = Path(config.run_dir) if config.run_dir else Path(config.out_root) / f"{config.eval_name}-{commit8}"
    if run_dir.exists() and any(run_dir.iterdir()):
        raise FileExistsError(f"{run_dir} exists; refusing a silent overwrite")
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "config.yaml").write_text(yaml.safe_dump(asdict(config), sort_keys=False))
    log_file = open(run_dir / "log.txt", "a", encoding="utf-8")

    def log(msg: str):
        line = f'[{datetime.now().strftime("%H:%M:%S")}] {msg}'
        print(line, flush=True)
        log_file.write(line + "\n")
        log_file.flush()

    device = resolve_device(config.device)
    dtype = _DTYPES[config.dtype]
    for t in config.tasks:
        if t["name"] not in TASKS:
            raise KeyError(f'unknown task {t["name"]!r}; registered: {sorted(TASKS)}')
    started = datetime.now().astimezone()
    t_start = time.perf_counter()
    log(f"eval {run_dir.name} | device {device} {config.dtype} | seed {config.seed} | "
        f"{len(config.subjects)} subjects x {len(config.tasks)} tasks")
    results = {t["name"]: {"args": t.get("args") or {}, "subjects": {}, "pairs": {}} for t in config.tasks}
    subjects_meta, labels = [], []
    for spec in config.subjects:
        subject = load_subject(spec, device, dtype)
        if subject.label in labels:
            raise ValueError(f"duplicate subject label {subject.label!r}")
        labels.append(subject.label)
        subjects_meta.append(subject.identity())
        log(f'subject {subject.label}: sha {subject.sha256[:8]} | {subject.meta["model_name"]} '
            f"{subject.param_count / 1e6:.1f}M")
        for t in config.tasks:
            name, args = t["name"], t.get("args") or {}
            t0 = time.perf_counter()
            res: TaskResult = TASKS[name](EvalCtx(subject, name, config.seed, device, dtype, log), **args)
            elapsed = time.perf_counter() - t0
            if res.samples:
                sdir = run_dir / "samples" / name
                sdir.mkdir(parents=True, exist_ok=True)
                with open(sdir / f"{subject.label}.jsonl", "w", encoding="utf-8") as f:
                    for row in res.samples:
                        f.write(json.dumps(row, ensure_ascii=False) + "\n")
            results[name]["subjects"][subject.label] = {
                "scalars": res.scalars, "items": {k: [round(float(x), 6) for x in v] for k, v in res.items.items()},
                "witness": res.witness, "elapsed_s": round(elapsed, 1)}
            log(f"task {name} on {subject.label} done in {elapsed:.1f}s")
            _write_json(run_dir / "results.json", results)
        del subject
        gc.collect()
        if device.type == "cuda":
            torch.cuda.empty_cache()
    ref = labels[0]
    for name, block in results.items():
        ref_items = block["subjects"][ref]["items"]
        for label in labels[1:]:
            other = block["subjects"][label]["items"]
            block["pairs"][label] = {k: paired(ref_items[k], other[k], n_boot=config.n_boot, seed=config.seed)
                                     for k in ref_items if k in other and len(other[k]) == len(ref_items[k])}
    meta = {"created": started.isoformat(timespec="seconds"),
            "finished": datetime.now().astimezone().isoformat(timespec="seconds"),
            "elapsed_s": round(time.perf_counter() - t_start, 1), "code": code, "torch": torch.__version__,
            "device": str(device), "dtype": config.dtype, "seed": config.seed, "reference": ref,
            "subjects": subjects_meta, "tasks": config.tasks}
    _write_json(run_dir / "meta.json", meta)
    _write_json(run_dir / "results.json", results)
    if config.registry_dir:
        rdir = Path(config.registry_dir)
        rdir.mkdir(parents=True, exist_ok=True)
        _write_json(rdir / f"{run_dir.name}.json", {"config": asdict(config), "meta": meta, "results": results})
    log(f'done in {meta["elapsed_s"]}s: {run_dir}')
    log_file.close()
    return run_dir


def main(argv=None):
    p = argparse.ArgumentParser(description="vagus_b200 evaluation")
    p.add_argument("recipe")
    p.add_argument("overrides", nargs="*")
    a = p.parse_args(argv)
    evaluate(EvalConfig.from_yaml(a.recipe, a.overrides))


if __name__ == "__main__":
    sys.exit(main())
