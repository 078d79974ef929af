"""Training observability: what the trainer reports each step, how it is
reduced, and where it goes.

The trainer calls ``Monitor.observe`` once per optimizer step with that
step's device scalars (mean loss, the z-loss term or None, the global grad
norm).  Nothing is read back on those calls: the scalars are stacked into a
device-side window, and on CUDA an event marks the step's end on the stream.
At a log event (every ``log_interval`` steps, and on ``final``) the window is
packed into one (steps x 3) tensor, averaged over the ranks by a single
all-reduce and copied to the host once; step time is the device time between
the window's first and last events, so host-side stalls between launches do
not enter it.

Probes are ``fn(ctx: MetricCtx) -> {name: float}``.  The built-in fast probes
(``FAST_METRICS``) run at every log event; the slow ones (``SLOW_METRICS``,
every ``slow_interval`` steps) reduce over every parameter: per optimizer
group the parameter norm and the norm of the next update (AdamW from its
moments, Muon from the orthogonalised update's closed form), all groups in
ONE vector reduced over the shard group of the FSDP mesh (DTensor local
shards) -- not one collective per tensor.  A model adds its own probes with
``metric_hooks() -> {"fast": [...], "slow": [...]}``; they read ``ctx.model``
and ``ctx.last_batch`` and run inside ``ctx.slow_context()`` when given
(FSDP: parameters unsharded).

Scalar names are the reference's (``loss``, ``loss_ema``, ``loss_ce``,
``loss_z``, ``lr``, ``grad_norm``, ``grad_norm_step_ratio``, ``tokens``,
``tokens_per_s``, ``step_ms``, ``mfu``, ``max_mem_gb``, ``pnorm/<group>``,
``pnorm/embedding``, ``upd_ratio/<group>``) so dashboards and the run
registry read runs of either framework; ``loss`` and ``grad_norm`` are the
log step's values and ``loss_ema`` is updated once per log event, as there.
``loss_window`` (mean over the window's steps) is added.

Parity: reference ``infra/train/metrics.py:59-267`` (MetricCtx, metric_core,
metric_throughput, metric_param_norms, metric_update_ratio, Monitor).
"""

from __future__ import annotations

import json
import math
import time
from contextlib import nullcontext
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.distributed as dist

try:
    from torch.distributed.tensor import DTensor
except ImportError:  # pragma: no cover
    DTensor = ()  # type: ignore


@dataclass
class MetricCtx:
    """What probes may read.  Static per run: ``model`` (unwrapped),
    ``optimizer``, ``world_size``, ``device_type``, ``param_count``,
    ``peak_tflops`` (per device; enables ``mfu``), ``attn_flops_per_tok``.
    Per log event: ``loss``, ``loss_ema``, ``z_term``, ``lr``,
    ``grad_norm``, ``prev_grad_norm``, ``tokens_seen``, ``tokens_per_s``,
    ``step_ms``.  ``last_batch``: the latest input ids of this rank (probes
    that run the model); ``slow_context``: () -> context manager around the
    slow probes."""
    model: Any = None
    optimizer: Any = None
    world_size: int = 1
    device_type: str = "cpu"
    param_count: int = 0
    peak_tflops: float | None = None
    attn_flops_per_tok: float = 0.0
    loss: float = 0.0
    loss_ema: float | None = None
    z_term: float | None = None
    lr: float = 0.0
    grad_norm: float = 0.0
    prev_grad_norm: float = 0.0
    tokens_seen: int = 0
    tokens_per_s: float = 0.0
    step_ms: float = 0.0
    last_batch: Any = None
    slow_context: Any = None
    memo: dict = field(default_factory=dict)     # per log event, shared by probes (cleared by Monitor)


# ------------------------------------------------------------- fast probes --

def metric_core(c: MetricCtx) -> dict:
    """Loss terms, learning rate, gradient norm and its change since the
    previous log event, tokens seen.  With a z-loss, ``loss`` is the whole
    objective and ``loss_ce`` the part comparable across z settings."""
    out = {"loss": c.loss, "loss_ema": c.loss_ema, "lr": c.lr, "grad_norm": c.grad_norm, "tokens": c.tokens_seen}
    if c.z_term is not None:
        out.update(loss_z=c.z_term, loss_ce=c.loss - c.z_term)
    if c.prev_grad_norm:
        out["grad_norm_step_ratio"] = c.grad_norm / c.prev_grad_norm
    return out


def metric_throughput(c: MetricCtx) -> dict:
    """Tokens / s of the job, ms per step and -- with a per-device peak --
    model FLOPs utilisation by the 6N-plus-attention estimate."""
    out = {"tokens_per_s": c.tokens_per_s, "step_ms": c.step_ms}
    if c.peak_tflops:
        per_device = (6.0 * c.param_count + c.attn_flops_per_tok) * c.tokens_per_s / c.world_size
        out["mfu"] = per_device / (c.peak_tflops * 1e12)
    if c.device_type == "cuda":
        out["max_mem_gb"] = torch.cuda.max_memory_allocated() / 1e9
    return out


# ------------------------------------------------------------- slow probes --

class _GroupSums:
    """Per-name squared sums over parameters that may be FSDP shards.

    Sharded tensors contribute their local shard; their totals need a sum
    over the mesh dimension they are sharded on, done for every name at once
    by ``reduce()``.  Replicated tensors (identical on every rank) are added
    after that reduction, so they count once."""

    def __init__(self, device):
        self.device = device
        self.names: list[str] = []
        self.sharded: list[list[torch.Tensor]] = []
        self.local: list[list[torch.Tensor]] = []
        self.groups: list = []           # in parameter order, identical on every rank

    def _slot(self, name: str) -> int:
        if name not in self.names:
            self.names.append(name)
            self.sharded.append([])
            self.local.append([])
        return self.names.index(name)

    def add(self, name: str, t: torch.Tensor, like=None) -> None:
        """``t``, or -- with ``like`` a DTensor -- ``t`` as this rank's shard
        of a tensor sharded like ``like``."""
        i = self._slot(name)
        ref = like if like is not None else t
        if isinstance(ref, DTensor):
            for dim, pl in enumerate(ref.placements):
                g = ref.device_mesh.get_group(dim)
                if pl.is_shard() and all(g is not h for h in self.groups):
                    self.groups.append(g)
            self.sharded[i].append(t.to_local() if isinstance(t, DTensor) else t)
        else:
            self.local[i].append(t)

    @staticmethod
    def _sq(ts: list[torch.Tensor]) -> torch.Tensor | None:
        ts = [t.detach().float() for t in ts if t.numel()]
        if not ts:
            return None
        return torch.stack(torch._foreach_norm(ts)).square().sum()

    def reduce(self) -> dict[str, float]:
        if not self.names:
            return {}
        zero = torch.zeros((), device=self.device)
        vec = torch.stack([s if (s := self._sq(ts)) is not None else zero for ts in self.sharded])
        for g in self.groups:           # one collective per sharding group (one group for FSDP / HSDP)
            dist.all_reduce(vec, group=g)
        loc = torch.stack([s if (s := self._sq(ts)) is not None else zero for ts in self.local])
        return dict(zip(self.names, (vec + loc).tolist()))


def _adam_direction(p_state: dict, group: dict) -> torch.Tensor:
    """The next AdamW step's direction m_hat / (sqrt(v_hat) + eps)."""
    b1, b2 = group["betas"]
    step = p_state["step"]
    t = float(step.full_tensor() if isinstance(step, DTensor) else step)
    m, v = p_state["exp_avg"], p_state["exp_avg_sq"]
    if isinstance(m, DTensor):
        m, v = m.to_local(), v.to_local()
    return (m.float() / (1 - b1 ** t)) / ((v.float() / (1 - b2 ** t)).sqrt() + group["eps"])


def _slow_sums(c: MetricCtx) -> tuple[dict, dict]:
    """(squared sums by name, Muon update squared norms by group) for the
    parameter-norm and update-ratio probes: reduced together, once per log
    event (memoised in ``c.memo``)."""
    if "slow_sums" in c.memo:
        return c.memo["slow_sums"]
    from ..optim.muon import lr_scale
    groups = c.optimizer.param_groups
    dev = next((p.device for g in groups for p in g["params"]), torch.device("cpu"))
    sums = _GroupSums(dev)
    muon_sq: dict[str, float] = {}
    state = c.optimizer.state
    for g in groups:
        name = g["name"]
        for p in g["params"]:
            sums.add(f"p/{name}", p)
            s = state.get(p)
            if not s:
                continue                   # before the first step
            if "exp_avg" in s:
                sums.add(f"a/{name}", _adam_direction(s, g), like=p)
            elif "momentum_buffer" in s:   # orthogonalised: ||O||_F^2 ~ min(m, n)
                rows, cols = p.shape
                muon_sq[name] = muon_sq.get(name, 0.0) + (g["lr"] * lr_scale((rows, cols), g["lr_adjust"])) ** 2 \
                    * min(rows, cols)
    emb = getattr(c.model, "embedding", None)
    if emb is not None:
        sums.add("embedding", emb.weight)
    c.memo["slow_sums"] = (sums.reduce(), muon_sq)
    return c.memo["slow_sums"]


def metric_param_norms(c: MetricCtx) -> dict:
    """L2 norm of each optimizer group's parameters and of the embedding."""
    sq, _ = _slow_sums(c)
    out = {f"pnorm/{k[2:]}": math.sqrt(v) for k, v in sq.items() if k.startswith("p/")}
    if "embedding" in sq:
        out["pnorm/embedding"] = math.sqrt(sq["embedding"])
    return out


def metric_update_ratio(c: MetricCtx) -> dict:
    """||next update|| / ||parameters|| per group at the current lr (weight
    decay left out): AdamW from the post-step moments, Muon from the
    orthogonalised update's closed form (exact up to the Newton-Schulz
    singular-value spread)."""
    sq, muon_sq = _slow_sums(c)
    out = {}
    for g in c.optimizer.param_groups:
        name = g["name"]
        upd = muon_sq.get(name, 0.0) + g["lr"] ** 2 * sq.get(f"a/{name}", 0.0)
        pn = sq.get(f"p/{name}", 0.0)
        if pn > 0 and upd > 0:
            out[f"upd_ratio/{name}"] = math.sqrt(upd / pn)
    return out


FAST_METRICS = [metric_core, metric_throughput]
SLOW_METRICS = [metric_param_norms, metric_update_ratio]


# ----------------------------------------------------------------- monitor --

class Monitor:
    """Cadence, device-side step window, reductions and sinks (metrics.jsonl,
    TensorBoard, console).  Build it on every rank -- a log event is a
    collective, and the cadence (``step % log_interval``) is identical
    everywhere; pass the sinks (``tb_dir``, ``jsonl_path``, a rank-gated
    ``log_fn``) on the main rank only.  Whether ``z`` is given must not
    change between steps."""

    def __init__(self, ctx: MetricCtx, tokens_per_step: int, steps_total: int, *, log_interval: int,
                 slow_interval: int, tb_dir=None, meta_text: str | None = None, log_fn: Callable = print,
                 print_every: int = 10, fast=FAST_METRICS, slow=SLOW_METRICS, jsonl_path=None):
        self.ctx = ctx
        self.tokens_per_step = tokens_per_step
        self.steps_total = steps_total
        self.log_interval = max(1, int(log_interval))
        self.slow_interval = max(1, int(slow_interval))
        self.log_fn = log_fn
        self.print_every = print_every
        self.fast, self.slow = list(fast), list(slow)
        self.history: list[dict] = []
        self._window: list[torch.Tensor] = []
        self._events: list = []
        self._prev_event = None
        self._t_host = time.perf_counter()
        self._steps_since = 0
        self.jsonl = open(jsonl_path, "a", encoding="utf-8") if jsonl_path is not None else None
        self.writer = None
        if tb_dir is not None:
            try:
                from torch.utils.tensorboard import SummaryWriter
                self.writer = SummaryWriter(tb_dir)
                if meta_text:
                    self.writer.add_text("meta", meta_text)
            except Exception as e:  # noqa: BLE001 -- TensorBoard is optional
                log_fn(f"[warn] tensorboard unavailable ({e}); scalars go to metrics.jsonl only")

    def _park(self, loss, grad_norm, z) -> None:
        """Stack this step's scalars on the device (no host read)."""
        loss_t = loss if torch.is_tensor(loss) else torch.tensor(float(loss))
        dev = loss_t.device
        z_t = (z if torch.is_tensor(z) else torch.tensor(float(z), device=dev)) if z is not None \
            else torch.zeros((), device=dev)
        g_t = grad_norm if torch.is_tensor(grad_norm) else torch.tensor(float(grad_norm), device=dev)
        self._window.append(torch.stack([loss_t.detach().float().reshape(()), z_t.detach().float().reshape(()),
                                         g_t.detach().float().reshape(()).to(dev)]))
        if dev.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._events.append(ev)
        self._steps_since += 1

    def _drain(self) -> tuple[list[list[float]], float]:
        """(per-step [loss, z, grad norm] averaged over ranks, ms per step)."""
        packed = torch.stack(self._window)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(packed, op=dist.ReduceOp.AVG)      # the grad norm is global: averaging keeps it
        rows = packed.tolist()                                # the one host read of the window
        now = time.perf_counter()
        if len(self._events) >= 2 and self._prev_event is not None:
            ms = self._prev_event.elapsed_time(self._events[-1]) / self._steps_since
        else:
            ms = (now - self._t_host) * 1e3 / self._steps_since
        self._prev_event = self._events[-1] if self._events else None
        self._t_host = now
        self._window, self._events, self._steps_since = [], [], 0
        return rows, ms

    def observe(self, step: int, loss: torch.Tensor, grad_norm, tokens_seen: int, final: bool = False,
                z: torch.Tensor | None = None):
        self._park(loss, grad_norm, z)
        if step % self.log_interval and not final:
            return
        n = self._steps_since
        rows, ms = self._drain()
        c = self.ctx
        c.loss, z_last, g_last = rows[-1]
        c.z_term = z_last if z is not None else None
        c.loss_ema = c.loss if c.loss_ema is None else 0.9 * c.loss_ema + 0.1 * c.loss
        c.prev_grad_norm, c.grad_norm = c.grad_norm, g_last
        c.lr = c.optimizer.param_groups[0]["lr"]
        c.tokens_seen = tokens_seen
        c.step_ms = ms
        c.tokens_per_s = self.tokens_per_step / (ms / 1e3) if ms > 0 else 0.0
        c.memo.clear()
        scalars = {"loss_window": sum(r[0] for r in rows) / n}
        for fn in self.fast:
            scalars |= fn(c)
        if step % self.slow_interval == 0:
            with (c.slow_context() if c.slow_context is not None else nullcontext()):
                for fn in self.slow:
                    scalars |= fn(c)
        self._emit(step, scalars, final)

    def _emit(self, step: int, scalars: dict, final: bool) -> None:
        row = {"step": step, **{k: v for k, v in scalars.items() if isinstance(v, (int, float))}}
        self.history.append(row)
        if self.jsonl is not None:
            self.jsonl.write(json.dumps(row) + "\n")
            self.jsonl.flush()
        if self.writer is not None:
            for k, v in row.items():
                if k != "step":
                    self.writer.add_scalar(k, v, step)
        if step % (self.log_interval * self.print_every) == 0 or final:
            c = self.ctx
            self.log_fn(f"step {step:>7,}/{self.steps_total:,} | loss {c.loss:.4f} (ema {c.loss_ema:.4f}) | "
                        f"lr {c.lr:.2e} | gnorm {c.grad_norm:.2f} | {c.step_ms:.0f} ms/step | "
                        f"{c.tokens_per_s / 1e6:.3f} Mtok/s")

    def close(self):
        if self.jsonl is not None:
            self.jsonl.close()
            self.jsonl = None
        if self.writer is not None:
            self.writer.close()
            self.writer = None
