"""Evaluation: a recipe of subjects (checkpoints) x tasks, run on the
Decodable protocol through the Generator, recorded with paired statistics
(``main.evaluate``); the shared item sampler and scorer live in ``core``."""
from .core import Draws, EvalCtx, Subject, TaskResult, log_probs  # noqa: F401
from .main import EvalConfig, evaluate  # noqa: F401
