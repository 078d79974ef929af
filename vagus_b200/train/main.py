"""Pretraining entry point: ``vagus-b200-train recipe.yaml [key=value ...]``.

Design contract (same recipe keys and run-directory layout as the reference):

* model / optimizer / schedule are picked by name + args dict;
* resume is the primary path: the run directory holds the resolved config,
  witnessed metadata, TensorBoard events and checkpoints, and restarting the
  same command continues exactly (loader state + RNG + optimizer restored);
* the stop condition is a token budget; the schedule lives on progress
  fractions;
* parallelism is one knob, ``shard_size``: 1 = DDP, N = FSDP2 over a 2-D
  (replicate, shard) mesh (HSDP when N < world).

Cooperative stop: SIGTERM / SIGUSR1 set a flag, ``SLURM_JOB_END_TIME`` sets a
deadline; every step the ranks all-reduce MAX a (stop, want_recent,
past_deadline) vector so they all take the same collective branch, write the
recent checkpoint and exit 0.  Checkpoints rotate recent -> recent-prev
before an atomic write; resume tries recent, recent-prev, then the newest
permanent checkpoint.

Parity: reference ``infra/train/main.py:72-759``.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import time
from contextlib import nullcontext
from dataclasses import asdict, dataclass, field
from datetime import datetime
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import yaml
from torch import nn

from .. import ops
from ..config import apply_overrides, load_yaml
from ..data.loader import TokenStore, WindowLoader
from ..models import build_model
from ..models.io import export_slim
from ..models.losses import make_ce
from ..optim import build_optimizer
from ..parallel import (DTYPES, LMLoss, apply_fsdp, build_mesh, clip_grad_norm, optimizer_members, wrap_ddp,
                        reduce_replicated, setup_distributed, unsharded, unwrap)
from ..utils import atomic_write, git_state
from .metrics import FAST_METRICS, SLOW_METRICS, MetricCtx, Monitor
from .schedule import build_schedule

try:
    from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_model_state_dict,
                                                         get_optimizer_state_dict, set_model_state_dict,
                                                         set_optimizer_state_dict)
    _FULL = StateDictOptions(full_state_dict=True, cpu_offload=True)
    _FROM_RANK0 = StateDictOptions(full_state_dict=True, broadcast_from_rank0=True)
except ImportError:  # pragma: no cover
    _FULL = _FROM_RANK0 = None


@dataclass
class TrainConfig:
    run_name: str
    data_dir: str
    model_name: str = "TransformerPP"
    model_args: dict = field(default_factory=dict)
    optimizer_name: str = "adamw"
    optimizer_args: dict = field(default_factory=lambda: dict(lr=3.0e-4, betas=(0.9, 0.95), weight_decay=0.1))
    schedule_name: str = "cosine"
    schedule_args: dict = field(default_factory=lambda: dict(warmup=0.01, min_ratio=0.05))
    data_shards: list | None = None
    context_len: int = 2048
    batch_size: int = 8
    grad_accum_steps: int = 1
    world_size: int = 1
    global_batch_tokens: int | None = None
    train_tokens: int = 1_000_000_000
    seed: int = 42
    shard_size: int = 1
    fsdp_param_dtype: str = "bfloat16"
    fsdp_reduce_dtype: str = "float32"
    fsdp_reshard_after_forward: bool = True
    fsdp_comm: str = "nvlink"          # FSDP2 all-gather / reduce-scatter: our NVLink kernels or "nccl"
    ddp_comm: str = "nvlink"           # DDP bucket all-reduce: our NVLink kernel (a DDP comm hook) or "nccl"
    grad_clip: float | None = 1.0
    z_loss: float | None = None
    ce_impl: str = "liger"
    ce_chunk_rows: int = 4096
    device: str = "auto"
    dtype: str = "bfloat16"
    compile: bool = True
    tf32: bool = True
    out_root: str = "runs"
    run_dir: str | None = None
    log_interval: int = 10
    slow_interval: int = 100
    permanent_ckpt_interval: int | None = None
    recent_ckpt_minutes: float = 30.0
    deadline_margin_s: float | None = 1200.0
    peak_tflops: float | None = None

    @classmethod
    def from_yaml(cls, path: str | Path, overrides=()) -> "TrainConfig":
        """A train recipe may include a pure model recipe via ``model_recipe:``
        (relative to the train recipe); the two may not both define the model.
        Unknown keys raise ``TypeError``."""
        path = Path(path)
        raw = load_yaml(path)
        if "model_recipe" in raw:
            mpath = (path.parent / raw.pop("model_recipe")).resolve()
            model = load_yaml(mpath)
            if not set(model) <= {"model_name", "model_args"}:
                raise ValueError(f"{mpath} is not a pure model recipe")
            if set(model) & set(raw):
                raise ValueError("model defined in both train and model recipe")
            raw |= model
        return cls(**apply_overrides(raw, overrides))


# ---------------------------------------------------------------- checkpoints --

def _strip(sd: dict, prefix: str) -> dict:
    return {k[len(prefix):] if k.startswith(prefix) else k: v for k, v in sd.items()}


def gather_state(model, optimizer, is_fsdp: bool) -> tuple[dict, dict, str]:
    """(model state, optimizer state, format); a collective under FSDP, where
    the dicts come back filled on rank 0 only."""
    if not is_fsdp:
        return unwrap(model).state_dict(), optimizer.state_dict(), "native"
    msd = _strip(get_model_state_dict(model, options=_FULL), "module.")
    osd = get_optimizer_state_dict(model, optimizer_members(optimizer), options=_FULL)
    return msd, osd, "dcp"


def load_state(model, optimizer, state: dict, is_fsdp: bool) -> None:
    if not is_fsdp:
        fmt = state.get("optimizer_format", "native")
        assert fmt == "native", f"{fmt} checkpoint cannot be loaded into the DDP regime"
        unwrap(model).load_state_dict(state["model"])
        optimizer.load_state_dict(state["optimizer"])
        return
    if state:
        fmt = state.get("optimizer_format", "native")
        assert fmt == "dcp", f"{fmt} checkpoint cannot be loaded into the FSDP regime"
    msd = {"module." + k: v for k, v in state.get("model", {}).items()}
    set_model_state_dict(model, msd, options=_FROM_RANK0)
    set_optimizer_state_dict(model, optimizer_members(optimizer), optim_state_dict=state.get("optimizer", {}),
                             options=_FROM_RANK0)


def save_checkpoint(run_dir: Path, kind: str, step: int, tokens_seen: int, model, optimizer, loader,
                    config: TrainConfig, is_fsdp: bool = False, is_main: bool = True):
    """Write a checkpoint from rank 0.  Every rank of a distributed job leaves
    only when the file is on disk: the others wait at a host barrier, so the
    next step's collectives never start while rank 0 is still writing (a
    multi-second skew the cross-GPU waits would otherwise have to absorb)."""
    msd, osd, fmt = gather_state(model, optimizer, is_fsdp)
    path = _write_checkpoint(run_dir, kind, step, tokens_seen, msd, osd, fmt, loader, config) if is_main else None
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    return path


def _write_checkpoint(run_dir: Path, kind: str, step: int, tokens_seen: int, msd, osd, fmt: str, loader,
                      config: TrainConfig) -> Path:
    state = {
        "step": step, "tokens_seen": tokens_seen, "model_name": config.model_name,
        "model_args": config.model_args,
        "tokenizer": {k: loader.store.manifest["tokenizer"][k] for k in ("id", "sha256")},
        "model": msd, "optimizer": osd, "optimizer_format": fmt, "loader": loader.state_dict(),
        "rng": {"torch": torch.get_rng_state(),
                "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None,
                "numpy": np.random.get_state()},
        "config": asdict(config),
    }
    path = run_dir / ("recent.pt" if kind == "recent" else f"ckpt-{step:08d}.pt")
    if kind == "recent" and path.exists():
        os.replace(path, run_dir / "recent-prev.pt")
    atomic_write(path, lambda f: torch.save(state, f))
    return path


def resume_candidates(run_dir: Path) -> list[Path]:
    """Checkpoints to resume from, best first: recent.pt, recent-prev.pt, then
    the permanent checkpoints newest first."""
    out = [run_dir / n for n in ("recent.pt", "recent-prev.pt") if (run_dir / n).exists()]
    return out + sorted(run_dir.glob("ckpt-*.pt"), reverse=True)


def find_resume(run_dir: Path) -> Path | None:
    c = resume_candidates(run_dir)
    return c[0] if c else None


def load_first_readable(cands: list[Path], log=print) -> tuple[Path, dict]:
    """The first candidate that loads; an unreadable file (truncated, corrupt)
    is reported and the next one is tried."""
    for p in cands:
        try:
            return p, torch.load(p, map_location="cpu", weights_only=False)
        except Exception as e:  # noqa: BLE001 -- any failure to read means: try the older file
            log(f"checkpoint {p.name} is unreadable ({type(e).__name__}: {e}); trying the next")
    raise RuntimeError(f"no readable checkpoint among {[p.name for p in cands]}")


# ------------------------------------------------------------------- training --

class StepRunner:
    """One optimizer step: ``grad_accum_steps`` micro-batches pulled from an
    iterator of host (x, y) batches, copied to the device (non-blocking from
    pinned memory), forward + fused CE + backward (DDP: gradient sync only on
    the last micro-step; FSDP: the root module computes the loss), the
    replicated-parameter reduction, clipping and the optimizer update.
    Returns (mean loss, mean z term or None, grad norm) as device tensors --
    nothing here synchronises with the host."""

    def __init__(self, model, optimizer, ce_fn, device, *, grad_accum_steps: int = 1, grad_clip=1.0,
                 is_fsdp: bool = False, is_dist: bool = False, replicate_size: int = 1, autocast=None, mesh=None):
        self.model = model
        self.optimizer = optimizer
        self.ce_fn = ce_fn
        self.device = device
        self.accum = grad_accum_steps
        self.grad_clip = grad_clip
        self.is_fsdp = is_fsdp
        self.is_dist = is_dist
        self.replicate_size = replicate_size
        self.autocast = autocast if autocast is not None else nullcontext()
        self.mesh = mesh
        self.head_weight = unwrap(model).head.weight
        self.last_batch = None

    def step(self, batches):
        model, ce_fn = self.model, self.ce_fn
        self.optimizer.zero_grad(set_to_none=True)
        loss_acc = torch.zeros((), device=self.device)
        z_acc = torch.zeros((), device=self.device) if ce_fn.tracks_z else None
        for micro in range(self.accum):
            x, y = next(batches)
            x = x.to(self.device, non_blocking=True)
            y = y.to(self.device, non_blocking=True)
            last = micro == self.accum - 1
            if self.is_fsdp:
                if self.replicate_size > 1:
                    model.set_requires_all_reduce(last)
                with self.autocast:
                    loss = model(x, y)
                    (loss / self.accum).backward()
            else:
                sync = model.no_sync() if self.is_dist and not last else nullcontext()
                with sync, self.autocast:
                    hidden = model(x, return_hidden=True)
                    loss = ce_fn(hidden, self.head_weight, y)
                    (loss / self.accum).backward()
            loss_acc += loss.detach()
            if z_acc is not None:
                z_acc += ce_fn.last_z
            self.last_batch = x
        if self.is_fsdp:
            reduce_replicated(model, self.mesh)
        grad_norm = clip_grad_norm(model, self.grad_clip)
        self.optimizer.step()
        return loss_acc / self.accum, (None if z_acc is None else z_acc / self.accum), grad_norm


_STOP = False


def _stop_handler(_signum, _frame):
    global _STOP
    _STOP = True


def request_stop() -> None:
    """Ask a running ``train()`` to stop at the next step boundary (what the
    signal handlers do; also usable from a test or a host thread)."""
    global _STOP
    _STOP = True


def resolve_run_dir(config: TrainConfig, code: dict | None = None) -> Path:
    """The run's directory: ``run_dir`` when the recipe sets it, else
    ``<out_root>/<run_name>-<commit8>`` (the code version is part of a run's
    identity).  Batch scripts call this to find the run they re-queue."""
    if config.run_dir:
        return Path(config.run_dir)
    code = git_state() if code is None else code
    return Path(config.out_root) / f"{config.run_name}-{(code['commit'] or 'nogit')[:8]}"


def train(config: TrainConfig, teardown: bool = True):
    global _STOP
    _STOP = False
    rank, world, device, is_dist = setup_distributed(config.device)
    is_main = rank == 0
    if world != config.world_size:
        raise ValueError(f"launched with world_size={world} but the recipe declares world_size={config.world_size}. "
                         "The data order depends on the card count, so this would be a different experiment.")
    declared = config.world_size * config.batch_size * config.grad_accum_steps * config.context_len
    if config.global_batch_tokens is not None and declared != config.global_batch_tokens:
        raise ValueError(f"world*batch*accum*ctx = {declared:,} does not match the declared "
                         f"global_batch_tokens = {config.global_batch_tokens:,}")
    mesh = build_mesh(config.shard_size, device, world)
    is_fsdp = mesh is not None
    replicate_size = mesh.size(0) if mesh is not None else 1

    def log(*a):
        if is_main:
            print(f'[{datetime.now().strftime("%H:%M:%S")}]', *a, flush=True)

    if hasattr(signal, "SIGUSR1"):
        try:
            signal.signal(signal.SIGTERM, _stop_handler)
            signal.signal(signal.SIGUSR1, _stop_handler)
        except ValueError:   # not the main thread (library use)
            pass
    deadline = None
    if config.deadline_margin_s is not None and os.environ.get("SLURM_JOB_END_TIME"):
        deadline = float(os.environ["SLURM_JOB_END_TIME"]) - config.deadline_margin_s

    torch.manual_seed(config.seed)
    np.random.seed(config.seed)
    if config.tf32 and device.type == "cuda":
        torch.backends.cuda.matmul.allow_tf32 = True
        torch.backends.cudnn.allow_tf32 = True

    code = git_state()
    run_dir = resolve_run_dir(config, code)
    resume_from = find_resume(run_dir) if run_dir.exists() else None
    if run_dir.exists() and resume_from is None and any(run_dir.iterdir()):
        raise FileExistsError(f"{run_dir} exists without checkpoints; refusing a silent overwrite")

    store = TokenStore(config.data_dir, shards=config.data_shards)
    loader = WindowLoader(store, config.context_len, config.batch_size, seed=config.seed, rank=rank, world_size=world,
                          pin_memory=device.type == "cuda")
    tokens_per_step = world * config.batch_size * config.grad_accum_steps * config.context_len
    steps_total = int(config.train_tokens) // tokens_per_step
    assert steps_total > 0

    amp_dtype = DTYPES[config.dtype]
    assert amp_dtype is not torch.float16, "fp16 (GradScaler) path not implemented"
    if is_fsdp and device.type == "cpu" and amp_dtype is torch.float32 and config.fsdp_param_dtype != "float32":
        # CUDA's linear kernels take an fp32 input against bf16 weights; the CPU ops do not
        raise ValueError(f"on CPU, dtype=float32 needs fsdp_param_dtype=float32 (got {config.fsdp_param_dtype}); "
                         "bf16 FSDP parameters pair with dtype=bfloat16 (autocast)")
    autocast = torch.autocast(device.type, dtype=amp_dtype) if amp_dtype is not torch.float32 else nullcontext()
    ce_fn = make_ce(config.ce_impl, z_loss=config.z_loss or 0.0, chunk_rows=config.ce_chunk_rows,
                    compute_dtype=amp_dtype if amp_dtype is not torch.float32 else None)

    model: nn.Module = build_model(config.model_name, config.model_args).to(device)
    param_count = sum(p.numel() for p in model.parameters())
    params_by_group = {k: sum(p.numel() for p in v) for k, v in model.param_groups().items()}
    if is_fsdp:
        model = LMLoss(model, ce_fn)
        apply_fsdp(model, mesh, config.fsdp_param_dtype, config.fsdp_reduce_dtype, config.fsdp_reshard_after_forward,
                   comm=config.fsdp_comm if device.type == "cuda" else "nccl")
    elif is_dist:
        model = wrap_ddp(model, device, config.ddp_comm if device.type == "cuda" else "nccl")
    optimizer = build_optimizer(config.optimizer_name, unwrap(model), config.optimizer_args)
    sched = build_schedule(config.schedule_name, config.schedule_args)

    layout = (f"HSDP mesh {tuple(mesh.shape)} (replicate, shard)" if mesh is not None
              else "DDP" if is_dist else "single")
    log(f"run {run_dir.name} | device {device} x{world} [{layout}] | {param_count:,} params | "
        f"data {store.total_tokens:,} tokens ({len(store.entries)} shards)")
    log(f"plan: {steps_total:,} steps x {tokens_per_step:,} tokens/step")

    if is_main and resume_from is None:
        run_dir.mkdir(parents=True, exist_ok=True)
        (run_dir / "config.yaml").write_text(yaml.safe_dump(asdict(config), sort_keys=False))
        (run_dir / "meta.json").write_text(json.dumps({
            "created": datetime.now().astimezone().isoformat(timespec="seconds"),
            "code": code, "world_size": world, "shard_size": config.shard_size, "device": str(device),
            "torch": torch.__version__, "config": asdict(config),
            "data": {"dir": str(Path(config.data_dir).resolve()), "source": store.manifest["source"],
                     "tokenizer": {k: store.manifest["tokenizer"][k] for k in ("id", "sha256")},
                     "total_tokens": store.total_tokens, "shards": [e["file"] for e in store.entries]},
            "derived": {"steps_total": steps_total, "tokens_per_step": tokens_per_step, "param_count": param_count,
                        "params_by_group": params_by_group, "windows": loader.window_count,
                        "batches_per_epoch": loader.batches_per_epoch},
        }, indent=2))

    step, tokens_seen = 0, 0
    if resume_from is not None:
        state: dict = {}
        if is_main or not is_fsdp:
            resume_from, state = load_first_readable(resume_candidates(run_dir), log)
            assert state["config"]["model_args"] == config.model_args, "checkpoint model_args differ from config"
        load_state(model, optimizer, state, is_fsdp)
        small = [{k: state[k] for k in ("step", "tokens_seen", "loader", "rng")} if state else None]
        if is_fsdp:
            dist.broadcast_object_list(small, src=0)
        rest = small[0]
        loader.load_state_dict(rest["loader"])
        torch.set_rng_state(rest["rng"]["torch"].cpu())
        if rest["rng"]["cuda"] is not None and torch.cuda.is_available():
            torch.cuda.set_rng_state_all([s.cpu() for s in rest["rng"]["cuda"]])
        np.random.set_state(rest["rng"]["numpy"])
        step, tokens_seen = rest["step"], rest["tokens_seen"]
        del state, rest
        log(f"resumed from {resume_from.name} at step {step:,}")

    ctx = MetricCtx(model=unwrap(model), optimizer=optimizer, world_size=world, device_type=device.type,
                    param_count=param_count, peak_tflops=config.peak_tflops,
                    attn_flops_per_tok=unwrap(model).attn_flops_per_token(config.context_len),
                    slow_context=(lambda: unsharded(model, autocast if config.fsdp_param_dtype != "float32" else None))
                    if is_fsdp else None)
    hooks = getattr(unwrap(model), "metric_hooks", dict)()
    monitor = Monitor(ctx, tokens_per_step, steps_total, log_interval=config.log_interval,
                      slow_interval=config.slow_interval, fast=FAST_METRICS + list(hooks.get("fast", [])),
                      slow=SLOW_METRICS + list(hooks.get("slow", [])), tb_dir=run_dir / "tb" if is_main else None,
                      log_fn=log, jsonl_path=run_dir / "metrics.jsonl" if is_main else None)
    runner = StepRunner(model, optimizer, ce_fn, device, grad_accum_steps=config.grad_accum_steps,
                        grad_clip=config.grad_clip, is_fsdp=is_fsdp, is_dist=is_dist,
                        replicate_size=replicate_size, autocast=autocast, mesh=mesh)
    batches = iter(loader)
    model.train()
    last_recent = time.time()
    stopped_early = False
    try:
        while step < steps_total:
            step += 1
            mult = sched(step / steps_total)
            for g in optimizer.param_groups:
                g["lr"] = g["base_lr"] * mult
            loss_acc, z_acc, grad_norm = runner.step(batches)
            ctx.last_batch = runner.last_batch
            tokens_seen += tokens_per_step
            if device.type == "cuda":
                ops.check_error()
            now = time.time()
            want_recent = now - last_recent > config.recent_ckpt_minutes * 60
            past_deadline = deadline is not None and now > deadline
            flags = torch.tensor([float(_STOP), float(want_recent), float(past_deadline)], device=device)
            if is_dist:
                dist.all_reduce(flags, op=dist.ReduceOp.MAX)
            stop = bool(flags[0].item()) or bool(flags[2].item())
            want_recent = bool(flags[1].item())
            stopped_early = stopped_early or stop
            monitor.observe(step, loss_acc, grad_norm, tokens_seen, final=stop or step == steps_total, z=z_acc)
            if config.permanent_ckpt_interval and step % config.permanent_ckpt_interval == 0 and step < steps_total:
                p = save_checkpoint(run_dir, "permanent", step, tokens_seen, model, optimizer, loader, config,
                                    is_fsdp, is_main)
                log(f'permanent checkpoint: {p.name if p else ""}')
            if want_recent:
                save_checkpoint(run_dir, "recent", step, tokens_seen, model, optimizer, loader, config, is_fsdp,
                                is_main)
                last_recent = time.time()
                log(f"recent checkpoint at step {step:,}")
            if stop:
                why = "walltime deadline reached" if bool(flags[2].item()) else "stop signal received"
                log(f"{why} at step {step:,}; checkpointing and exiting")
                break
        kind = "recent" if stopped_early else "permanent"
        p = save_checkpoint(run_dir, kind, step, tokens_seen, model, optimizer, loader, config, is_fsdp, is_main)
        if is_main:
            log(f"final {kind} checkpoint: {p.name} | {tokens_seen / 1e9:.3f}B tokens seen")
            if kind == "permanent":
                export_slim(p, run_dir / "model-final.pt")
                log("wrote model-final.pt (slim)")
    finally:
        monitor.close()
        if is_dist and teardown:
            dist.destroy_process_group()
    return run_dir


def main(argv=None):
    ap = argparse.ArgumentParser(prog="vagus-b200-train")
    ap.add_argument("config", help="path to a TrainConfig yaml")
    ap.add_argument("overrides", nargs="*", help="key=value top-level field overrides")
    a = ap.parse_args(argv)
    train(TrainConfig.from_yaml(a.config, a.overrides))


if __name__ == "__main__":
    main()
