"""Evaluation: recipe -> subjects x tasks -> record, on the Decodable protocol."""
from .core import EvalCtx, Subject, TaskResult  # noqa: F401
from .main import EvalConfig, evaluate  # noqa: F401
