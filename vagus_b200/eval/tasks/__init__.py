"""Task registry: ``run(ctx, **args) -> TaskResult``; items must be drawn from
``ctx.rng()`` / ``ctx.torch_seed()`` only (identical across subjects)."""
from . import degeneration, holdout, recall_probe, saturation

TASKS = {"holdout": holdout.run, "degeneration": degeneration.run, "recall_probe": recall_probe.run,
         "saturation": saturation.run}
