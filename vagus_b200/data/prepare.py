"""Tokenisation stage: local source parquet -> ``vagus-tokens-v1`` shards.

One source parquet maps to one shard: ``NNN.npy`` (uint16 token stream,
per-document BOS, no EOS, documents in source order) and ``NNN.idx.npy``
(uint64 document start offsets, docs + 1 entries) plus ``manifest.json``
(format, tokenizer fingerprint, provenance, per-shard sha256, totals,
status).  Idempotent: shards already in the manifest are skipped, so a rerun
resumes and a longer source list extends the dataset; the identity blocks must
match an existing manifest.

Parity: reference ``infra/dataset/prepare.py:28-157`` (same format).
"""

from __future__ import annotations

import hashlib
import importlib
import json
import time
from array import array
from datetime import datetime
from pathlib import Path

import numpy as np

from ..utils import atomic_write, git_state

FORMAT = "vagus-tokens-v1"


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while chunk := f.read(1 << 24):
            h.update(chunk)
    return h.hexdigest()


def tokenize_texts(tok, texts) -> tuple[np.ndarray, np.ndarray]:
    """Texts -> (uint16 tokens, uint64 doc offsets) with the tokenizer's own
    special-token handling (BOS per document)."""
    buf = array("H")
    offsets = array("Q", [0])
    for enc in tok.encode_batch(list(texts)):
        buf.extend(enc.ids)
        offsets.append(len(buf))
    return np.frombuffer(buf, dtype=np.uint16), np.frombuffer(offsets, dtype=np.uint64)


def _tokenize_file(tok, src: Path, batch_rows: int):
    import pyarrow.parquet as pq
    toks, offs = [], [np.zeros(1, dtype=np.uint64)]
    base = 0
    for batch in pq.ParquetFile(src).iter_batches(batch_size=batch_rows, columns=["text"]):
        t, o = tokenize_texts(tok, batch.column("text").to_pylist())
        toks.append(t)
        offs.append(o[1:] + base)
        base += len(t)
    tokens = np.concatenate(toks) if toks else np.zeros(0, dtype=np.uint16)
    return tokens, np.concatenate(offs)


def write_shard(out_dir: Path, stem: str, source: str, tokens: np.ndarray, offsets: np.ndarray) -> dict:
    shard, idx = out_dir / f"{stem}.npy", out_dir / f"{stem}.idx.npy"
    atomic_write(shard, lambda f: np.save(f, tokens.astype(np.uint16)))
    atomic_write(idx, lambda f: np.save(f, offsets.astype(np.uint64)))
    return {"file": shard.name, "idx": idx.name, "source": source, "tokens": int(len(tokens)),
            "docs": int(len(offsets) - 1), "sha256": sha256_file(shard)}


def _update_totals(manifest: dict, sources: list[str]) -> None:
    manifest["total_tokens"] = sum(s["tokens"] for s in manifest["shards"])
    manifest["total_docs"] = sum(s["docs"] for s in manifest["shards"])
    have = {s["source"] for s in manifest["shards"]}
    manifest["status"] = "complete" if all(s in have for s in sources) else "building"


def prepare(sources: list[Path], provenance: dict, out_dir, tokenizer_id: str = "mistral32k",
            batch_rows: int = 1000, tokenizer=None, fingerprint: str | None = None) -> Path:
    """Tokenise ``sources`` (order defines the stream) into ``out_dir``."""
    if tokenizer is None:
        tok_mod = importlib.import_module(f"vagus_b200.tokenizers.{tokenizer_id}")
        tok, fp = tok_mod.load(), tok_mod.fingerprint()
    else:
        tok, fp = tokenizer, fingerprint or "unknown"
    assert tok.get_vocab_size() <= 1 << 16, "uint16 shard format requires vocab <= 65536"
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    manifest_path = out_dir / "manifest.json"
    tokenizer_block = {"id": tokenizer_id, "sha256": fp, "vocab_size": tok.get_vocab_size(),
                       "convention": "per-doc BOS prefix, no EOS, docs concatenated in source order"}
    if manifest_path.exists():
        manifest = json.loads(manifest_path.read_text())
        for key, expect in (("format", FORMAT), ("source", provenance), ("tokenizer", tokenizer_block)):
            if manifest[key] != expect:
                raise ValueError(f"out_dir holds a different dataset: {key} mismatch")
    else:
        manifest = {"format": FORMAT, "status": "building",
                    "created": datetime.now().astimezone().isoformat(timespec="seconds"), "source": provenance,
                    "tokenizer": tokenizer_block, "dtype": "uint16", "files": [], "shards": [], "total_tokens": 0,
                    "total_docs": 0, "code": git_state()}
    done = {s["source"] for s in manifest["shards"]
            if (out_dir / s["file"]).exists() and (out_dir / s["idx"]).exists()}
    manifest["files"] = [src.name for src in sources]
    names = [src.name for src in sources]
    for src in sources:
        if src.name in done:
            continue
        t0 = time.perf_counter()
        tokens, offsets = _tokenize_file(tok, src, batch_rows)
        entry = write_shard(out_dir, src.stem, src.name, tokens, offsets)
        manifest["shards"] = sorted([s for s in manifest["shards"] if s["source"] != src.name] + [entry],
                                    key=lambda s: s["source"])
        _update_totals(manifest, names)
        atomic_write(manifest_path, lambda f: f.write(json.dumps(manifest, indent=2).encode()))
        dt = time.perf_counter() - t0
        print(f"{src.name}: {entry['tokens']:,} tokens, {entry['docs']:,} docs in {dt:.0f}s")
    _update_totals(manifest, names)
    atomic_write(manifest_path, lambda f: f.write(json.dumps(manifest, indent=2).encode()))
    return manifest_path


def synthetic_store(out_dir, tokens: int, vocab: int, *, seed: int = 0, shards: int = 1, doc_len: int = 0,
                    bos: int | None = None) -> Path:
    """A ``vagus-tokens-v1`` store of uniform-random tokens (benchmarks,
    tests).  ``doc_len`` > 0 inserts a ``bos`` token every ``doc_len`` tokens."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    entries = []
    per = tokens // shards
    lo = 2 if vocab > 2 else 0
    for i in range(shards):
        arr = rng.integers(lo, vocab, size=per, dtype=np.int64).astype(np.uint16)
        offs = [0]
        if doc_len and bos is not None:
            arr[::doc_len] = bos
            offs = list(range(0, per, doc_len))
        offs.append(per)
        entries.append(write_shard(out_dir, f"{i:03d}", f"synthetic-{i:03d}", arr, np.asarray(offs, dtype=np.uint64)))
    manifest = {"format": FORMAT, "status": "complete", "source": {"name": "synthetic", "seed": seed},
                "tokenizer": {"id": "synthetic", "sha256": "0" * 64, "vocab_size": vocab,
                              "convention": "uniform random ids"},
                "dtype": "uint16", "files": [e["source"] for e in entries], "shards": entries,
                "total_tokens": per * shards, "total_docs": sum(e["docs"] for e in entries)}
    (out_dir / "manifest.json").write_text(json.dumps(manifest, indent=2))
    return out_dir / "manifest.json"
