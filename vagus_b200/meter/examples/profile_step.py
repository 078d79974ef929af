"""Where a training step's time goes: one model's forward + backward +
optimizer step under torch.profiler, the top ops, a Chrome trace, and (on
CUDA) device time grouped by kernel family (GEMM, attention, delta-rule
recurrence, conv, norms / pointwise, CE, optimizer, collectives, other).

    python -m vagus_b200.meter.examples.profile_step --recipe recipe/model/lax1_340M.yaml --batch 8 --seq 4096
    python -m vagus_b200.meter.examples.profile_step --model GDNLM --args '{"dim": 256, ...}'

Parity: reference ``infra/meter/examples/bench_kda_kernel.py`` (``bench_model`` /
``profile_model``: a model's training step timed and profiled).
"""

from __future__ import annotations

import argparse
import json

import torch

from ..profiling import family  # noqa: F401  (re-exported: kernel-name families)


def build(a):
    from ...models import build_model
    if a.recipe:
        from ...config import load_yaml
        rec = load_yaml(a.recipe)
        name, margs = rec["model_name"], rec["model_args"]
    else:
        name, margs = a.model, json.loads(a.args)
    return name, margs, build_model(name, margs)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--recipe", default=None, help="a model recipe yaml (model_name, model_args)")
    ap.add_argument("--model", default="GDNLM")
    ap.add_argument("--args", default="{}", help="model_args as JSON (without --recipe)")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--optimizer", default="muon", choices=["muon", "adamw"])
    ap.add_argument("--out", default="profile-output")
    a = ap.parse_args(argv)
    from ...models.losses import make_ce
    from ...optim import build_optimizer
    from ...train.main import StepRunner
    from ..profiling import device_split, profile_variants, render_split
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    name, margs, model = build(a)
    model = model.to(dev)
    vocab = int(margs["vocab_size"])
    ce = make_ce("fused" if dev.type == "cuda" else "full", z_loss=1e-4)
    opt_args = dict(lr=2e-3, adamw=dict(lr=1e-3)) if a.optimizer == "muon" else dict(lr=1e-3)
    opt = build_optimizer(a.optimizer, model, opt_args)
    autocast = torch.autocast(dev.type, dtype=torch.bfloat16) if dev.type == "cuda" else None
    runner = StepRunner(model, opt, ce, dev, grad_accum_steps=1, grad_clip=1.0, autocast=autocast)
    g = torch.Generator().manual_seed(0)
    t = torch.randint(0, vocab, (a.batch, a.seq + 1), generator=g).to(dev)
    batch = (t[:, :-1], t[:, 1:])

    def step():
        loss, _z, _g = runner.step(iter([batch]))
        return loss

    traces = profile_variants({name: step}, steps=a.steps, warmup=a.warmup, out_dir=a.out, device=dev)
    if dev.type != "cuda" or not traces:
        return {"traces": {k: str(v) for k, v in traces.items()}}
    # device time by family, from a second, quiet profile
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            step()
        torch.cuda.synchronize()
    split = device_split(prof, a.steps)
    print(f"\ndevice time per step by kernel family ({sum(split['families_ms'].values()):.1f} ms):")
    print(render_split(split))
    return {"traces": {k: str(v) for k, v in traces.items()}, **split}


if __name__ == "__main__":
    main()
