"""LR schedules on run progress in [0, 1], returning a multiplier of the peak
lr: ``cosine`` (warmup then cosine to a floor), ``linear`` (warmup then
linear decay), ``wsd`` (warmup, stable, linear cooldown over the last
``decay`` fraction).  Validated at build time.

Parity: reference ``infra/train/schedule.py:12-49``.
"""

from __future__ import annotations

import math
from functools import partial
from typing import Callable


def cosine(progress: float, *, warmup: float = 0.01, min_ratio: float = 0.0) -> float:
    if progress < warmup:
        return progress / warmup
    p = (progress - warmup) / (1 - warmup)
    return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * p))


def linear(progress: float, *, warmup: float = 0.01, min_ratio: float = 0.05) -> float:
    if progress < warmup:
        return progress / warmup
    p = (progress - warmup) / (1 - warmup)
    return 1 + (min_ratio - 1) * p


def wsd(progress: float, *, warmup: float = 0.01, decay: float = 0.2, min_ratio: float = 0.0) -> float:
    if progress < warmup:
        return progress / warmup
    if progress < 1 - decay:
        return 1.0
    p = (progress - (1 - decay)) / decay
    return 1 + (min_ratio - 1) * p


SCHEDULES = {"cosine": cosine, "linear": linear, "wsd": wsd}


def build_schedule(name: str, args: dict) -> Callable[[float], float]:
    fn = partial(SCHEDULES[name], **args)
    for p in (0.0, 0.5, 1.0):
        fn(p)
    return fn
