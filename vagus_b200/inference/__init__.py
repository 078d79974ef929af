"""Generation: one stateful Generator over the Decodable protocol."""
from .generator import Generator  # noqa: F401
from .sampling import SamplingConfig, sample  # noqa: F401

__all__ = ["Generator", "SamplingConfig", "sample"]
