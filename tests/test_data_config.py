"""Token store, window loader (order, rank interleave, resume, fingerprint,
prefetch), data preparation, config loader and utilities — CPU."""

import json
import os

import numpy as np
import pytest
import torch

from vagus_b200.config import apply_overrides, load_yaml, parse_value
from vagus_b200.data.loader import TokenStore, WindowLoader
from vagus_b200.data.prepare import synthetic_store, tokenize_texts, write_shard
from vagus_b200.utils import atomic_write, git_state, infer_device, infer_dtype


@pytest.fixture()
def store(tmp_path):
    synthetic_store(tmp_path / "tok", tokens=40_000, vocab=500, seed=3, shards=2, doc_len=97, bos=1)
    return TokenStore(tmp_path / "tok")


def _batches(loader, n):
    it = iter(loader)
    return [next(it) for _ in range(n)]


def test_store_windows_and_docs(store):
    assert len(store.shard_tokens) == 2 and sum(store.shard_tokens) == 40_000
    w = store.read_window(0, 10, 50)
    assert w.shape == (50,) and w.dtype == np.uint16
    offs = store.doc_offsets(0)
    assert offs[0] == 0 and offs[-1] == store.shard_tokens[0]
    doc = store.doc(0, 1)
    assert doc[0] == 1 and len(doc) == offs[2] - offs[1]


def test_loader_is_deterministic_and_shapes(store):
    a = _batches(WindowLoader(store, 64, 4, seed=7, prefetch=0), 5)
    b = _batches(WindowLoader(store, 64, 4, seed=7, prefetch=0), 5)
    for (xa, ya), (xb, yb) in zip(a, b):
        assert xa.shape == (4, 64) and ya.shape == (4, 64)
        assert torch.equal(xa, xb) and torch.equal(ya, yb)
        assert torch.equal(xa[:, 1:], ya[:, :-1])          # targets are the inputs shifted by one
    c = _batches(WindowLoader(store, 64, 4, seed=8, prefetch=0), 1)
    assert not torch.equal(a[0][0], c[0][0])


def test_ranks_partition_the_global_batch(store):
    single = _batches(WindowLoader(store, 64, 4, seed=1, prefetch=0, world_size=1), 4)
    r0 = _batches(WindowLoader(store, 64, 2, seed=1, prefetch=0, rank=0, world_size=2), 4)
    r1 = _batches(WindowLoader(store, 64, 2, seed=1, prefetch=0, rank=1, world_size=2), 4)
    rows = lambda bs: {tuple(x.tolist()) for b in bs for x in b[0]}      # noqa: E731
    assert not rows(r0) & rows(r1)


def test_resume_continues_the_sequence(store):
    full = _batches(WindowLoader(store, 64, 4, seed=2, prefetch=0), 6)
    ld = WindowLoader(store, 64, 4, seed=2, prefetch=0)
    it = iter(ld)
    for _ in range(3):
        next(it)
    state = ld.state_dict()
    ld2 = WindowLoader(store, 64, 4, seed=2, prefetch=0)
    ld2.load_state_dict(state)
    rest = _batches(ld2, 3)
    for (x, y), (xf, yf) in zip(rest, full[3:]):
        assert torch.equal(x, xf) and torch.equal(y, yf)
    other = WindowLoader(store, 32, 4, seed=2, prefetch=0)
    with pytest.raises(Exception):
        other.load_state_dict(state)


def test_prefetch_matches_synchronous(store):
    a = _batches(WindowLoader(store, 64, 4, seed=5, prefetch=0), 4)
    b = _batches(WindowLoader(store, 64, 4, seed=5, prefetch=3), 4)
    for (xa, _), (xb, _) in zip(a, b):
        assert torch.equal(xa, xb)


def test_tokenize_and_write_shard(tmp_path):
    class Tok:
        def encode_batch(self, texts):
            class E:
                def __init__(self, ids):
                    self.ids = ids
            return [E([5 + len(w) for w in t.split()]) for t in texts]

        def token_to_id(self, t):
            return 1
    toks, offs = tokenize_texts(Tok(), ["a bb ccc", "dddd"])
    assert offs[0] == 0 and offs[-1] == len(toks)
    entry = write_shard(tmp_path, "000", "unit", toks.astype(np.uint16), offs.astype(np.uint64))
    assert (tmp_path / "000.npy").exists() and entry["tokens"] == len(toks)


def test_yaml_overrides_and_values(tmp_path):
    p = tmp_path / "r.yaml"
    p.write_text("lr: 1e-4\nmodel_args:\n  dim: 64\n  la_fused: false\nname: x\n")
    raw = load_yaml(p)
    assert isinstance(raw["lr"], float) and raw["lr"] == 1e-4
    raw = apply_overrides(raw, ["model_args.la_fused=true", "lr=3e-3", "name=y", "steps=10"])
    assert raw["model_args"] == {"dim": 64, "la_fused": True}
    assert raw["lr"] == 3e-3 and raw["name"] == "y" and raw["steps"] == 10
    assert parse_value("[1, 2]") == [1, 2] and parse_value("null") is None


def test_utils(tmp_path):
    f = tmp_path / "a" / "b.json"
    f.parent.mkdir()
    atomic_write(f, lambda fh: fh.write(json.dumps({"k": 1}).encode()))
    assert json.loads(f.read_text()) == {"k": 1}
    assert not [x for x in os.listdir(f.parent) if x != "b.json"]
    g = git_state()
    assert set(g) >= {"commit", "dirty"}
    t = torch.zeros(2, dtype=torch.bfloat16)
    assert infer_device((t,), {}).type == "cpu" and infer_dtype((t,), {}) == torch.bfloat16


def test_every_recipe_loads_and_builds():
    """Each committed train recipe (with its model recipe) parses, keeps its
    declared global batch, and builds its model (on the meta device)."""
    from pathlib import Path
    from vagus_b200.models import build_model
    from vagus_b200.train.main import TrainConfig
    recipes = sorted((Path(__file__).resolve().parents[1] / "recipe" / "train").glob("*.yaml"))
    assert recipes
    for f in recipes:
        c = TrainConfig.from_yaml(f)
        if c.global_batch_tokens is not None:
            assert c.world_size * c.batch_size * c.grad_accum_steps * c.context_len == c.global_batch_tokens, f
        with torch.device("meta"):
            build_model(c.model_name, c.model_args)


def test_console_scripts_resolve():
    """Every console script of pyproject.toml names an importable callable."""
    import importlib
    import tomllib
    from pathlib import Path
    meta = tomllib.loads((Path(__file__).resolve().parents[1] / "pyproject.toml").read_text())
    scripts = meta["project"]["scripts"]
    assert {"vagus-b200-train", "vagus-b200-eval"} <= set(scripts)
    for target in scripts.values():
        mod, _, fn = target.partition(":")
        assert callable(getattr(importlib.import_module(mod), fn)), target
