"""Recipe loading shared by every entry point (train, eval, bench).

One YAML dialect and one override syntax:

* YAML 1.1 reads ``1e-4`` (no dot) as a string; the loader here registers an
  implicit float resolver so scientific notation without a dot is a float.
* ``key=value`` overrides are parsed as YAML values; a dotted key reaches one
  level into a dict-valued field (``model_args.chunk_size=32``).

Parity: reference ``infra/config.py:11-56``.
"""

from __future__ import annotations

import re
from pathlib import Path

import yaml

__all__ = ["RecipeLoader", "load_yaml", "parse_value", "apply_overrides"]

_SCI_FLOAT = re.compile(
    r"""^[-+]?(?:
        (?:\d+(?:\.\d*)?|\.\d+)(?:[eE][-+]?\d+)?
      | \d+[eE][-+]?\d+
    )$""",
    re.X,
)


class RecipeLoader(yaml.SafeLoader):
    """SafeLoader plus the scientific-notation float resolver."""


RecipeLoader.add_implicit_resolver("tag:yaml.org,2002:float", _SCI_FLOAT, list("-+0123456789."))


def load_yaml(path: str | Path) -> dict:
    with open(path, encoding="utf-8") as fh:
        return yaml.load(fh, RecipeLoader) or {}


def parse_value(text: str):
    """Value side of an override (``4``, ``float32``, ``[a, b]``, ``null``)."""
    return yaml.load(text, RecipeLoader)


def apply_overrides(raw: dict, overrides) -> dict:
    """Return a copy of ``raw`` with ``key=value`` strings applied."""
    out = dict(raw)
    for item in overrides:
        key, sep, value = item.partition("=")
        if not sep or not key:
            raise ValueError(f"override {item!r} is not key=value")
        outer, dot, inner = key.partition(".")
        if not dot:
            out[key] = parse_value(value)
            continue
        if not isinstance(out.get(outer), dict):
            raise ValueError(f"override {item!r}: {outer} is not a dict field")
        out[outer] = {**out[outer], inner: parse_value(value)}
    return out
