"""Paired comparison of two subjects on the same items: mean difference, a
percentile-bootstrap 95% interval and the fraction of items that improved.

Parity: reference ``infra/eval/pairs.py:8-22``.
"""

from __future__ import annotations

import numpy as np


def paired(ref, other, n_boot: int = 2000, seed: int = 0) -> dict:
    a, b = np.asarray(ref, dtype=np.float64), np.asarray(other, dtype=np.float64)
    assert a.shape == b.shape and a.ndim == 1 and len(a) > 0
    d = b - a
    n = len(d)
    means = d[np.random.default_rng(seed).integers(0, n, (n_boot, n))].mean(axis=1)
    return {"n": n, "mean_diff": float(d.mean()),
            "ci95": [float(np.quantile(means, 0.025)), float(np.quantile(means, 0.975))],
            "frac_positive": float((d > 0).mean())}
