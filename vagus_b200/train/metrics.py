"""Training observability owned end to end by ``Monitor``: cadence, the loss
EMA, throughput and MFU, per-group parameter norms and update ratios, model
hooks (``metric_hooks()``), TensorBoard scalars and console lines.

Hooks are ``fn(MetricCtx) -> dict``; FAST ones run every log interval, SLOW
ones every ``slow_interval`` steps (they touch every parameter).  ``observe``
all-reduces the reported loss, which is safe because the cadence decision is
identical on every rank.

Parity: reference ``infra/train/metrics.py:59-267``.
"""

from __future__ import annotations

import math
import json
import time
from contextlib import nullcontext
from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.distributed as dist

try:
    from torch.distributed.tensor import DTensor
except ImportError:  # pragma: no cover
    DTensor = ()  # type: ignore


def _scalar(t) -> float:
    if isinstance(t, DTensor):
        t = t.full_tensor()
    return float(t)


def _sum(parts) -> float:
    parts = list(parts)
    if not parts:
        return 0.0
    total = parts[0]
    for x in parts[1:]:
        total = total + x
    return _scalar(total)


@dataclass
class MetricCtx:
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


def metric_core(c: MetricCtx) -> dict:
    out = {"loss": c.loss, "loss_ema": c.loss_ema, "lr": c.lr, "grad_norm": c.grad_norm, "tokens": c.tokens_seen}
    if c.z_term is not None:
        out["loss_z"] = c.z_term
        out["loss_ce"] = c.loss - c.z_term
    if c.prev_grad_norm:
        out["grad_norm_step_ratio"] = c.grad_norm / c.prev_grad_norm
    return out


def metric_throughput(c: MetricCtx) -> dict:
    out = {"tokens_per_s": c.tokens_per_s, "step_ms": c.step_ms}
    if c.peak_tflops:
        flops_per_tok = 6 * c.param_count + c.attn_flops_per_tok
        out["mfu"] = flops_per_tok * c.tokens_per_s / c.world_size / (c.peak_tflops * 1e12)
    if c.device_type == "cuda":
        out["max_mem_gb"] = torch.cuda.max_memory_allocated() / 1e9
    return out


def metric_param_norms(c: MetricCtx) -> dict:
    out = {}
    for g in c.optimizer.param_groups:
        out[f"pnorm/{g['name']}"] = math.sqrt(_sum(p.detach().float().pow(2).sum() for p in g["params"]))
    emb = getattr(c.model, "embedding", None)
    if emb is not None:
        out["pnorm/embedding"] = math.sqrt(_scalar(emb.weight.detach().float().pow(2).sum()))
    return out


def metric_update_ratio(c: MetricCtx) -> dict:
    """||update|| / ||param|| per group: AdamW from its moments, Muon from the
    closed form of the orthogonalised update (weight decay ignored)."""
    out = {}
    state = c.optimizer.state
    for g in c.optimizer.param_groups:
        lr = g["lr"]
        upd_sq = 0.0
        adam_parts = []
        pnorm_sq = _sum(p.detach().float().pow(2).sum() for p in g["params"])
        for p in g["params"]:
            s = state.get(p)
            if not s:
                continue
            if "exp_avg" in s:
                b1, b2 = g["betas"]
                t = float(_scalar(s["step"]))
                m_hat = s["exp_avg"].float() / (1 - b1 ** t)
                v_hat = s["exp_avg_sq"].float() / (1 - b2 ** t)
                adam_parts.append((m_hat / (v_hat.sqrt() + g["eps"])).pow(2).sum())
            elif "momentum_buffer" in s:
                m, n = p.shape
                if g["lr_adjust"] == "rms":
                    upd_sq += (0.2 * lr) ** 2 * p.numel()
                else:
                    upd_sq += (lr * max(1.0, m / n) ** 0.5) ** 2 * min(m, n)
        if adam_parts:
            upd_sq += lr * lr * _sum(adam_parts)
        if pnorm_sq > 0 and upd_sq > 0:
            out[f"upd_ratio/{g['name']}"] = math.sqrt(upd_sq / pnorm_sq)
    return out


FAST_METRICS = [metric_core, metric_throughput]
SLOW_METRICS = [metric_param_norms, metric_update_ratio]


class Monitor:
    def __init__(self, ctx: MetricCtx, tokens_per_step: int, steps_total: int, *, log_interval: int,
                 slow_interval: int, tb_dir=None, meta_text: str | None = None, log_fn: Callable = print,
                 print_every: int = 10, fast=FAST_METRICS, slow=SLOW_METRICS, jsonl_path=None):
        self.ctx = ctx
        self.tokens_per_step = tokens_per_step
        self.steps_total = steps_total
        self.log_interval = log_interval
        self.slow_interval = slow_interval
        self.log_fn = log_fn
        self.print_every = print_every
        self.fast = fast
        self.slow = slow
        self.writer = None
        self.history: list[dict] = []
        # one JSON line per logged step (the run registry reads it)
        self.jsonl = open(jsonl_path, "a", encoding="utf-8") if jsonl_path is not None else None
        if tb_dir is not None:
            try:
                from torch.utils.tensorboard import SummaryWriter
                self.writer = SummaryWriter(tb_dir)
                if meta_text:
                    self.writer.add_text("meta", meta_text)
            except Exception as e:  # tensorboard is optional
                log_fn(f"[warn] tensorboard unavailable ({e}); scalars kept in memory only")
        self._t = time.perf_counter()

    def observe(self, step: int, loss: torch.Tensor, grad_norm, tokens_seen: int, final: bool = False,
                z: torch.Tensor | None = None):
        if step % self.log_interval != 0 and not final:
            return
        if dist.is_available() and dist.is_initialized():
            if z is not None:
                pack = torch.stack([loss, z])
                dist.all_reduce(pack, op=dist.ReduceOp.AVG)
                loss, z = pack[0], pack[1]
            else:
                dist.all_reduce(loss, op=dist.ReduceOp.AVG)
        c = self.ctx
        now = time.perf_counter()
        c.loss = float(loss)
        c.z_term = float(z) if z is not None else None
        c.loss_ema = c.loss if c.loss_ema is None else 0.9 * c.loss_ema + 0.1 * c.loss
        c.prev_grad_norm, c.grad_norm = c.grad_norm, float(grad_norm)
        c.lr = c.optimizer.param_groups[0]["lr"]
        c.tokens_seen = tokens_seen
        c.step_ms = (now - self._t) / self.log_interval * 1e3
        c.tokens_per_s = self.tokens_per_step * self.log_interval / (now - self._t)
        self._t = now
        scalars = {}
        for fn in self.fast:
            scalars |= fn(c)
        if step % self.slow_interval == 0:
            with (c.slow_context() if c.slow_context is not None else nullcontext()):
                for fn in self.slow:
                    scalars |= fn(c)
        row = {"step": step, **{k: v for k, v in scalars.items() if isinstance(v, (int, float))}}
        self.history.append(row)
        if self.jsonl is not None:
            self.jsonl.write(json.dumps(row) + "\n")
            self.jsonl.flush()
        if self.writer is not None:
            for k, v in scalars.items():
                self.writer.add_scalar(k, v, step)
        if step % (self.log_interval * self.print_every) == 0 or final:
            self.log_fn(f"step {step:>7,}/{self.steps_total:,} | loss {c.loss:.4f} (ema {c.loss_ema:.4f}) | "
                        f"lr {c.lr:.2e} | gnorm {c.grad_norm:.2f} | {c.tokens_per_s / 1e6:.2f} Mtok/s")

    def close(self):
        if self.jsonl is not None:
            self.jsonl.close()
            self.jsonl = None
        if self.writer is not None:
            self.writer.close()
