"""Task registry: a recipe's ``tasks: [{name, args}]`` selects by name and
passes ``args`` as keywords to ``run(ctx, **args) -> TaskResult``.  A task
draws its items through ``ctx.draws`` / ``ctx.rng`` / ``ctx.torch_seed``
only, so they are the same for every subject."""
from . import degeneration, holdout, recall_probe, saturation

TASKS = {"holdout": holdout.run, "degeneration": degeneration.run, "recall_probe": recall_probe.run,
         "saturation": saturation.run}
