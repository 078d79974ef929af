"""Evaluation entry point: ``vagus-b200-eval recipe.yaml [key=value ...]``.

An evaluation is a recipe of subjects (checkpoints) and tasks; the runner
resolves each subject once, runs every task on it, frees it, and moves on.
Tasks draw their items from (seed, task, salt) only, so after the last
subject every per-item array lines up across subjects, and each subject is
paired against the first (the reference) item by item: mean difference,
bootstrap 95 % interval, share of items that went up.

``EvalRecord`` owns the run directory -- ``config.yaml``, ``log.txt``,
``results.json`` (rewritten after every task, so a crash keeps what ran),
``samples/<task>/<label>.jsonl``, ``meta.json`` -- refuses a directory that
already holds files, and copies the whole record (config, meta, results)
to the registry directory when one is configured.

Record layout (kept identical to the reference, so records of the two
frameworks are read by the same tools): ``results.json`` maps task -> {args,
subjects: {label: {scalars, items (6 decimals), witness, elapsed_s}}, pairs:
{label: {item key: paired statistics}}}; ``meta.json`` holds created,
finished, elapsed_s, code, torch, device, dtype, seed, reference, subjects
(``Subject.identity()``) and tasks.

Parity: reference ``infra/eval/main.py`` (EvalConfig fields, subject specs,
the record files and their layout).
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
from ..data.prepare import sha256_file
from ..inference import Generator
from ..utils import atomic_write, git_state
from .core import EvalCtx, Subject, TaskResult
from .pairs import paired
from .tasks import TASKS

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@dataclass
class EvalConfig:
    """An eval recipe.  ``subjects``: checkpoint paths, run directories
    (their ``model-final.pt``) or dicts ``{ckpt | run, label, tokenizer_id,
    run_meta}`` (``run_meta``: the training run's meta.json when it does not
    sit beside the checkpoint); the first subject is the reference of the
    pairs.  ``tasks``: ``[{name, args}]`` with names from ``tasks.TASKS``."""
    eval_name: str
    subjects: list
    tasks: list
    device: str = "auto"
    dtype: str = "bfloat16"
    seed: int = 0
    out_root: str = "runs/eval"
    run_dir: str | None = None            # default: <out_root>/<eval_name>-<commit8>
    registry_dir: str | None = "registry/eval"
    n_boot: int = 2000

    @classmethod
    def from_yaml(cls, path, overrides=()) -> "EvalConfig":
        return cls(**apply_overrides(load_yaml(path), overrides))

    def validate(self) -> None:
        """Task names are registered and their arguments are accepted."""
        import inspect
        for t in self.tasks:
            fn = TASKS.get(t.get("name"))
            if fn is None:
                raise KeyError(f"unknown task {t.get('name')!r}; registered: {sorted(TASKS)}")
            params = inspect.signature(fn).parameters
            extra = set(t.get("args") or {}) - set(params) - {"ctx"}
            if extra:
                raise TypeError(f"task {t['name']}: unknown arguments {sorted(extra)}")


def resolve_device(name: str) -> torch.device:
    if name != "auto":
        return torch.device(name)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def load_subject(spec, device: torch.device, dtype: torch.dtype) -> Subject:
    """A subject spec -> Subject (generator, checkpoint record and hash, and
    the training run's meta.json when it is found)."""
    spec = {"ckpt": spec} if isinstance(spec, str) else dict(spec)
    src = Path(spec.get("ckpt") or spec["run"])
    ckpt = src / "model-final.pt" if src.is_dir() else src
    label = spec.get("label") or (src.name if src.is_dir() else src.stem)
    gen, meta = Generator.from_checkpoint(ckpt, device=device, dtype=dtype, tokenizer_id=spec.get("tokenizer_id"),
                                         with_meta=True)
    run_meta = None
    where = Path(spec["run_meta"]) if spec.get("run_meta") else ckpt.parent / "meta.json"
    if where.exists():
        rec = json.loads(where.read_text())
        is_train_meta = "config" in rec and "data" in rec
        if is_train_meta:
            run_meta = rec
        elif spec.get("run_meta"):
            raise ValueError(f"{where} is not the meta.json of a training run")
    return Subject(label=label, path=ckpt.resolve(), sha256=sha256_file(ckpt), meta=meta, generator=gen,
                   run_meta=run_meta)


class EvalRecord:
    """The files of one evaluation run."""

    def __init__(self, run_dir: Path, config: EvalConfig):
        if run_dir.exists() and any(run_dir.iterdir()):
            raise FileExistsError(f"{run_dir} already holds an evaluation; refusing to overwrite it")
        run_dir.mkdir(parents=True, exist_ok=True)
        self.dir = run_dir
        self.config = config
        (run_dir / "config.yaml").write_text(yaml.safe_dump(asdict(config), sort_keys=False))
        self._log = open(run_dir / "log.txt", "a", encoding="utf-8")
        self.results = {t["name"]: {"args": t.get("args") or {}, "subjects": {}, "pairs": {}} for t in config.tasks}
        self.labels: list[str] = []
        self.identities: list[dict] = []

    @staticmethod
    def _json(path: Path, obj) -> None:
        atomic_write(path, lambda f: f.write(json.dumps(obj, indent=2).encode()))

    def log(self, msg: str) -> None:
        line = f"[{datetime.now():%H:%M:%S}] {msg}"
        print(line, flush=True)
        self._log.write(line + "\n")
        self._log.flush()

    def add_subject(self, subject: Subject) -> None:
        if subject.label in self.labels:
            raise ValueError(f"two subjects are labelled {subject.label!r}")
        self.labels.append(subject.label)
        self.identities.append(subject.identity())

    def add_result(self, task: str, label: str, res: TaskResult, seconds: float) -> None:
        if res.samples:
            path = self.dir / "samples" / task / f"{label}.jsonl"
            path.parent.mkdir(parents=True, exist_ok=True)
            path.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in res.samples), encoding="utf-8")
        self.results[task]["subjects"][label] = {
            "scalars": res.scalars, "items": {k: [round(float(x), 6) for x in v] for k, v in res.items.items()},
            "witness": res.witness, "elapsed_s": round(seconds, 1)}
        self._json(self.dir / "results.json", self.results)

    def pair_all(self) -> None:
        """Every subject against the first, on the item arrays both have at
        the same length."""
        ref = self.labels[0]
        for task, block in self.results.items():
            base = block["subjects"][ref]["items"]
            for label in self.labels[1:]:
                other = block["subjects"][label]["items"]
                block["pairs"][label] = {k: paired(v, other[k], n_boot=self.config.n_boot, seed=self.config.seed)
                                         for k, v in base.items() if len(other.get(k, ())) == len(v)}
                head = [(k, p) for k, p in block["pairs"][label].items() if not k.startswith(("gold_", "copy_"))]
                self.log(f"{task}: {label} vs {ref}: " + " ".join(
                    f"{k} {p['mean_diff']:+.4f} [{p['ci95'][0]:+.4f}, {p['ci95'][1]:+.4f}]" for k, p in head[:6]))

    def close(self, meta: dict) -> None:
        self._json(self.dir / "meta.json", meta)
        self._json(self.dir / "results.json", self.results)
        if self.config.registry_dir:
            reg = Path(self.config.registry_dir)
            reg.mkdir(parents=True, exist_ok=True)
            self._json(reg / f"{self.dir.name}.json", {"config": asdict(self.config), "meta": meta,
                                                       "results": self.results})
            self.log(f"record copied to {reg / (self.dir.name + '.json')}")
        self._log.close()


def evaluate(config: EvalConfig) -> Path:
    config.validate()
    code = git_state()
    name = f"{config.eval_name}-{(code['commit'] or 'nogit')[:8]}"
    record = EvalRecord(Path(config.run_dir) if config.run_dir else Path(config.out_root) / name, config)
    device, dtype = resolve_device(config.device), DTYPES[config.dtype]
    started, t0 = datetime.now().astimezone(), time.perf_counter()
    record.log(f"eval {record.dir.name}: {len(config.subjects)} subjects x {len(config.tasks)} tasks on {device} "
               f"({config.dtype}), seed {config.seed}{' (code dirty)' if code.get('dirty') else ''}")
    for spec in config.subjects:
        subject = load_subject(spec, device, dtype)
        record.add_subject(subject)
        record.log(f"subject {subject.label}: {subject.path.name} sha {subject.sha256[:8]}, "
                   f"{subject.meta['model_name']} {subject.param_count / 1e6:.1f}M, step {subject.meta.get('step')}")
        for t in config.tasks:
            task, args = t["name"], t.get("args") or {}
            ts = time.perf_counter()
            res = TASKS[task](EvalCtx(subject, task, config.seed, device, dtype, record.log), **args)
            record.add_result(task, subject.label, res, time.perf_counter() - ts)
            record.log(f"task {task} on {subject.label}: {time.perf_counter() - ts:.1f}s")
        del subject
        gc.collect()
        if device.type == "cuda":
            torch.cuda.empty_cache()
    record.pair_all()
    meta = {"created": started.isoformat(timespec="seconds"),
            "finished": datetime.now().astimezone().isoformat(timespec="seconds"),
            "elapsed_s": round(time.perf_counter() - t0, 1), "code": code, "torch": torch.__version__,
            "device": str(device), "dtype": config.dtype, "seed": config.seed, "reference": record.labels[0],
            "subjects": record.identities, "tasks": config.tasks}
    record.close(meta)
    return record.dir


def main(argv=None):
    p = argparse.ArgumentParser(description="vagus_b200 evaluation: subjects x tasks -> record")
    p.add_argument("recipe")
    p.add_argument("overrides", nargs="*", help="key=value overrides (yaml values), e.g. device=cpu")
    a = p.parse_args(argv)
    evaluate(EvalConfig.from_yaml(a.recipe, a.overrides))


if __name__ == "__main__":
    sys.exit(main())
