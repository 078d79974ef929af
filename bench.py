"""Headline benchmark: training tokens/s of the 340M gated-DeltaNet LM
-- vocab 32000, d_model 1024, 24 layers, 4 heads x 256,
short conv 4, output gate, chunk 64, SwiGLU 2816, seq 4096, 0.5M tokens per
optimizer step (Muon + AdamW), synthetic uniform-random tokens, random init.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

For N > 1 launch one rank per GPU with torch.distributed.run (RANK /
LOCAL_RANK / WORLD_SIZE / MASTER_* come from the environment).  The global
batch stays 0.5M tokens at every N (strong scaling): each rank runs
128 / (N * micro) micro-batches of ``micro`` sequences per step.  The GDN and
hybrid configs train under FSDP2, Transformer++ under DDP (BASELINE config
#2); ``--parallelism`` overrides.

Measurement:
* ``value``: W untimed warm-up steps, then K steps bracketed by a barrier and
  torch.cuda.synchronize() on both sides, timed with CUDA events on the
  launching stream; the max over ranks.  Inputs are already on the device.
  Every step's working set is far larger than L2, so no explicit flush.
* ``e2e``: K more steps through the public StepRunner API with each step's
  tokens copied host -> device from pinned memory and the loss read back to
  the host every step; wall clock between barriers, max over ranks.
* ``clocks``: nvidia-smi sampled every 200 ms during the timed region.
* ``gpu_launches``: calls into the in-tree extension per step (each binding
  launches one kernel) x K, counted on an extra untimed step.

``--impl reference`` runs the reference (installed under baseline/_ref)
through its own public API and stock path: its model registry, fused CE,
Muon+AdamW factory, regional torch.compile, bf16 autocast, FSDP2 or DDP for
N > 1 as the config says.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from contextlib import nullcontext
from pathlib import Path

ROOT = Path(__file__).resolve().parent

CONFIGS = {
    # the headline benchmark: 340M GDN, FSDP2 + Muon
    "gdn340m": dict(
        model_name="GDNLM",
        model_args=dict(vocab_size=32000, dim=1024, layer_count=24, head_count=4, key_head_dim=256,
                        value_head_dim=256, ffn_hidden_dim=2816, short_conv_size=4, gate="scalar", delta=True,
                        chunk_size=64, context_len=4096, la_impl="auto"),
        seq=4096, global_tokens=524288, micro=16, label="340M GDN (4x256, chunk 64), FSDP2+Muon"),
    # 1.3B hybrid GDN/softmax 3:1, FSDP2 + sharded Muon
    "hybrid1.3b": dict(
        model_name="GDNLM",
        model_args=dict(vocab_size=32000, dim=2048, layer_count=24, head_count=8, key_head_dim=256,
                        value_head_dim=256, ffn_hidden_dim=5632, short_conv_size=4, gate="scalar", delta=True,
                        chunk_size=64, layer_pattern="gdn,gdn,gdn,softmax", softmax_head_dim=128,
                        context_len=4096, la_impl="auto"),
        seq=4096, global_tokens=1048576, micro=4, label="1.3B hybrid GDN/softmax 3:1"),
    # 340M hybrid KDA/softmax 3:1 (recipe/model/kda_hybrid_340M.yaml)
    "kda_hybrid340m": dict(
        model_name="GDNLM",
        model_args=dict(vocab_size=32000, dim=1024, layer_count=24, head_count=4, key_head_dim=128,
                        value_head_dim=256, ffn_hidden_dim=2816, short_conv_size=4, gate="vector", gate_rank=64,
                        delta=True, chunk_size=64, layer_pattern="gdn,gdn,gdn,softmax", softmax_head_dim=64,
                        softmax_rope=True, context_len=4096, la_impl="auto"),
        seq=4096, global_tokens=524288, micro=8, label="340M hybrid KDA/softmax 3:1"),
    # 340M Transformer++, AdamW
    "tpp340m": dict(
        model_name="TransformerPP",
        model_args=dict(vocab_size=32000, dim=1024, head_dim=64, context_len=4096, layer_count=24,
                        ffn_hidden_dim=2816),
        seq=4096, global_tokens=524288, micro=4, label="340M Transformer++", optimizer="adamw", parallelism="ddp"),
    # small shape for plumbing checks (not a headline number)
    "tiny": dict(
        model_name="GDNLM",
        model_args=dict(vocab_size=4096, dim=256, layer_count=2, head_count=2, key_head_dim=128, value_head_dim=128,
                        ffn_hidden_dim=704, gate="scalar", chunk_size=64, context_len=512),
        seq=512, global_tokens=16384, micro=8, label="tiny"),
}

# Configurations whose reference stock path faulted the GPU on this pool: they
# are not run again; each entry says what ran and how it failed.
REFERENCE_FAULTS = {
    "gdn340m": ("reference stock path (fla chunk_gated_delta_rule, head_dim 256) raised CUDA 'misaligned address' "
                "in fla prepare_wy_repr_bwd (Triton autotune) on B200; not re-run under the GPU-fault policy"),
    "hybrid1.3b": ("same fla chunk_gated_delta_rule backward at head_dim 256 as gdn340m, which faulted on B200; "
                   "not run under the GPU-fault policy"),
}

MUON = dict(lr=1.75e-3, momentum=0.95, weight_decay=0.1, lr_adjust="rms", ns_coeffs="polar_express",
            adamw=dict(lr=1.75e-3, betas=[0.9, 0.95], weight_decay=0.1))
ADAMW = dict(lr=3e-4, betas=[0.9, 0.95], weight_decay=0.1)


class ClockSampler:
    """nvidia-smi clock / throttle sampling in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        load = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def _synthetic(n_batches, micro, seq, vocab, seed, pin):
    import torch
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n_batches):
        t = torch.randint(0, vocab, (micro, seq + 1), generator=g)
        if pin:
            t = t.pin_memory()
        out.append((t[:, :-1], t[:, 1:]))
    return out


def _max_over_ranks(v: float, is_dist: bool) -> float:
    import torch
    import torch.distributed as dist
    if not is_dist:
        return v
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _count_launches(fn) -> int:
    """Calls into the in-tree extension made by ``fn()`` (one kernel each)."""
    from vagus_b200.ops import _core
    real = _core.native()
    counter = {"n": 0}
    skip = {"error_word", "reset_error"}

    class Proxy:
        def __getattr__(self, name):
            attr = getattr(real, name)
            if callable(attr) and name not in skip:
                def wrapped(*a, **k):
                    counter["n"] += 1
                    return attr(*a, **k)
                return wrapped
            return attr

    _core._C = Proxy()
    try:
        fn()
    finally:
        _core._C = real
    return counter["n"]


def run(args) -> dict:
    import torch
    import torch.distributed as dist
    rank, world, local = _dist_env()
    cfg = CONFIGS[args.config]
    is_dist = world > 1
    par = args.parallelism if args.parallelism != "auto" else cfg.get("parallelism", "fsdp")
    is_fsdp = is_dist and par == "fsdp"
    if is_dist:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"),
                                timeout=datetime.timedelta(seconds=600))
        if args.impl != "reference":
            sys.path.insert(0, str(ROOT))
            from vagus_b200.parallel.nvlink import set_peer_wait_seconds
            set_peer_wait_seconds(600)      # the kernels' cross-GPU waits end with the group's timeout
    dev = torch.device(f"cuda:{local}")
    torch.manual_seed(0)
    seq, micro = cfg["seq"], (args.micro or cfg["micro"])
    if args.global_tokens:
        cfg = dict(cfg, global_tokens=args.global_tokens)
    per_rank_seqs = cfg["global_tokens"] // seq // world
    micro = min(micro, per_rank_seqs)
    accum = per_rank_seqs // micro
    assert accum * micro * world * seq == cfg["global_tokens"], "global batch must split evenly"
    vocab = cfg["model_args"]["vocab_size"]
    opt_name = cfg.get("optimizer", "muon")
    opt_args = MUON if opt_name == "muon" else ADAMW

    if args.impl == "reference":
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        from infra.components.losses import make_ce
        from infra.models import build_model
        from infra.optimizer import build_optimizer
        from infra.train import main as ref_main
        model = build_model(cfg["model_name"], cfg["model_args"]).to(dev)
        if hasattr(model, "compile_blocks"):
            model.compile_blocks()
        ce = make_ce("liger", z_loss=1e-4, compute_dtype=torch.bfloat16)
        mesh = None
        if is_fsdp:
            mesh = ref_main.build_mesh(ref_main.TrainConfig(run_name="b", data_dir="", shard_size=world,
                                                            world_size=world), dev, world)
            model = ref_main.LMLoss(model, ce)
            ref_main.apply_fsdp(model, mesh, ref_main.TrainConfig(run_name="b", data_dir="", shard_size=world,
                                                                  world_size=world))
        elif is_dist:
            from torch.nn.parallel import DistributedDataParallel as DDP
            model = DDP(model, device_ids=[dev.index], output_device=dev.index)
        optimizer = build_optimizer(opt_name, ref_main.unwrap(model), json.loads(json.dumps(opt_args)))
        head = ref_main.unwrap(model).head.weight
        autocast = torch.autocast("cuda", dtype=torch.bfloat16)

        def step(batches):
            optimizer.zero_grad(set_to_none=True)
            acc = torch.zeros((), device=dev)
            for micro_i in range(accum):
                x, y = next(batches)
                x = x.to(dev, non_blocking=True)
                y = y.to(dev, non_blocking=True)
                sync = model.no_sync() if is_dist and not is_fsdp and micro_i < accum - 1 else nullcontext()
                with sync, autocast:
                    if is_fsdp:
                        loss = model(x, y)
                    else:
                        loss = ce(model(x, return_hidden=True), head, y)
                    (loss / accum).backward()
                acc += loss.detach()
            if is_fsdp:
                ref_main.reduce_replicated(model, mesh)
            ref_main.clip_grad_norm(model, 1.0)
            optimizer.step()
            return acc / accum
    else:
        sys.path.insert(0, str(ROOT))
        from vagus_b200 import ops
        from vagus_b200.models import build_model
        from vagus_b200.models.losses import make_ce
        from vagus_b200.optim import build_optimizer
        from vagus_b200.parallel import LMLoss, apply_fsdp, build_mesh, unwrap, wrap_ddp
        from vagus_b200.train.main import StepRunner
        ops.native()
        model = build_model(cfg["model_name"], cfg["model_args"]).to(dev)
        ce = make_ce("fused", z_loss=1e-4)
        mesh = None
        if is_fsdp:
            mesh = build_mesh(world, dev, world)
            model = LMLoss(model, ce)
            apply_fsdp(model, mesh, comm=args.comm)
        elif is_dist:
            model = wrap_ddp(model, dev, comm=args.comm)
        optimizer = build_optimizer(opt_name, unwrap(model), json.loads(json.dumps(opt_args)))
        runner = StepRunner(model, optimizer, ce, dev, grad_accum_steps=accum, grad_clip=1.0, is_fsdp=is_fsdp,
                            is_dist=is_dist, mesh=mesh)

        def step(batches):
            loss, _z, _g = runner.step(batches)
            return loss

    host = _synthetic(accum, micro, seq, vocab, seed=1000 + rank, pin=True)
    devb = [(x.to(dev), y.to(dev)) for x, y in host]

    def cycle(src):
        while True:
            yield from src

    dev_iter = cycle(devb)
    t0 = time.time()
    for _ in range(args.warmup):
        step(dev_iter)
    torch.cuda.synchronize()
    warm_s = time.time() - t0

    launches = None
    if args.impl != "reference":
        torch.cuda.synchronize()
        launches = _count_launches(lambda: step(dev_iter))
        torch.cuda.synchronize()

    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
    if is_dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        loss = step(dev_iter)
    ev1.record()
    torch.cuda.synchronize()
    if is_dist:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = _max_over_ranks(ms, is_dist)
    final_loss = float(loss.item())

    # end to end: host batches (pinned) -> device every micro-step, loss to host every step
    host_iter = cycle(host)
    if is_dist:
        dist.barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        loss = step(host_iter)
        float(loss.item())
    torch.cuda.synchronize()
    if is_dist:
        dist.barrier()
    e2e_ms = _max_over_ranks((time.perf_counter() - w0) * 1e3 / args.steps, is_dist)
    clocks = sampler.stop() if rank == 0 else None

    # the optimizer step alone (Muon: momentum, Newton-Schulz, its collectives),
    # on the gradients of the last step; device time, max over ranks
    optimizer.step()
    if is_dist:
        dist.barrier()
    torch.cuda.synchronize()
    o0, o1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    o0.record()
    for _ in range(3):
        optimizer.step()
    o1.record()
    torch.cuda.synchronize()
    opt_ms = _max_over_ranks(o0.elapsed_time(o1) / 3, is_dist)

    # opt-in (--exposed-comm, FSDP on our NVLink collectives): the same steps
    # with the FSDP2 all-gathers / reduce-scatters switched off; the
    # difference to the timed step is the communication the compute did not hide
    exposed = None
    if args.exposed_comm and is_fsdp and args.impl != "reference" and args.comm == "nvlink":
        from vagus_b200.parallel import nvlink as nvl
        nvl.set_dry_run(True)
        for _ in range(2):
            step(dev_iter)
        dist.barrier()
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record()
        for _ in range(args.steps):
            step(dev_iter)
        d1.record()
        torch.cuda.synchronize()
        dist.barrier()
        nvl.set_dry_run(False)
        dry_ms = _max_over_ranks(d0.elapsed_time(d1) / args.steps, is_dist)
        exposed = {"ms_per_step_without_fsdp_collectives": round(dry_ms, 2), "exposed_ms": round(ms - dry_ms, 2),
                   "pct_of_step": round(100.0 * (ms - dry_ms) / ms, 2),
                   "covers": "FSDP2 parameter all-gathers and gradient reduce-scatters"}

    tokens_per_step = cfg["global_tokens"]
    value = tokens_per_step / (ms / 1e3)
    e2e = tokens_per_step / (e2e_ms / 1e3)
    h2d = accum * micro * (seq * 2) * 8     # x and y int64 per micro-step, this rank
    out = {
        "metric": "train tokens/s/box 340M GDN (BASELINE config #3)" if args.config == "gdn340m"
        else f"train tokens/s/box ({cfg['label']})",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic uniform-random tokens, random init",
        "config": {"model": cfg["label"], "global_batch": cfg["global_tokens"], "seq_len": seq,
                   "micro_batch": micro, "grad_accum": accum,
                   "parallelism": f"{par}{world}" if world > 1 else "single",
                   "collectives": ("nccl" if args.impl == "reference" else args.comm) if world > 1 else None,
                   "optimizer": opt_name, "l2": "no flush: every step's working set is >> 126 MB L2"},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4},
        "gpu_launches": None if launches is None else launches * args.steps,
        "clocks": clocks, "final_loss": round(final_loss, 4), "warmup_s": round(warm_s, 1),
        "max_mem_gb": round(torch.cuda.max_memory_allocated() / 1e9, 1),
        "optimizer_step_ms": round(opt_ms, 2),
    }
    if exposed is not None:
        out["exposed_comm"] = exposed
    if args.impl == "reference":
        out["impl"] = "reference"
    if is_dist:
        dist.barrier()
        dist.destroy_process_group()
    return out if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--comm", default="nvlink", choices=["nvlink", "nccl"],
                    help="collectives of our arm (FSDP2 all-gather / reduce-scatter, DDP all-reduce): "
                         "NVLink peer-to-peer kernels or NCCL")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="gdn340m")
    ap.add_argument("--micro", type=int, default=0, help="sequences per micro-batch (0: the config's default)")
    ap.add_argument("--global-tokens", type=int, default=0,
                    help="tokens per optimizer step (0: the config's; a diagnostic, not the headline batch)")
    ap.add_argument("--parallelism", choices=["auto", "ddp", "fsdp"], default="auto",
                    help="N > 1: DDP or FSDP2 (auto: the config's, DDP for tpp340m as BASELINE config #2)")
    ap.add_argument("--exposed-comm", action="store_true",
                    help="N > 1: also time the steps with the FSDP2 collectives off and report the exposed share")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference" and not (ROOT / "baseline" / "_ref" / "infra").exists():
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    if args.impl == "reference" and args.config in REFERENCE_FAULTS:
        print(json.dumps({"impl": "reference", "unavailable": REFERENCE_FAULTS[args.config]}))
        return
    out = run(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
