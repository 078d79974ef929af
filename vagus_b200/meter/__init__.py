"""meter: a small performance measurement toolkit (``bench``, ``compare``,
``profile_variants``; ``meter.dist`` for per-rank benches)."""
from .compare import compare, render_table  # noqa: F401
from .core import BenchResult, bench, synchronize  # noqa: F401
from .profiling import profile_variants  # noqa: F401
