"""Training: the trainer entry point, the per-step runner, LR schedules and
the metrics monitor."""
from .main import StepRunner, TrainConfig, train  # noqa: F401
