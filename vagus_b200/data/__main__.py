"""``python -m vagus_b200.data {download,tokenize,synthetic}``.

download   pinned FineWeb-Edu parquet prefix (network)
tokenize   parquet -> vagus-tokens-v1 shards (no network, idempotent)
synthetic  a store of uniform-random tokens of a given size (benchmarks)

Parity: reference ``infra/dataset/__main__.py:21-82``.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from . import fineweb_edu
from .prepare import prepare, synthetic_store


def _local_sources(sample: str, count: int, out_dir: Path) -> list[Path]:
    dest = fineweb_edu.default_dest() / "sample" / sample
    have = {p.name: p for p in dest.glob("*.parquet")}
    done = set()
    mp = out_dir / "manifest.json"
    if mp.exists():
        m = json.loads(mp.read_text())
        done = {s["source"] for s in m["shards"] if (out_dir / s["file"]).exists() and (out_dir / s["idx"]).exists()}
    names = sorted(set(have) | done)
    if len(names) < count:
        raise SystemExit(f"{len(names)} sources known, need {count} -- run `download` first")
    return [have.get(n, dest / n) for n in names[:count]]


def main(argv=None):
    p = argparse.ArgumentParser(prog="python -m vagus_b200.data")
    sub = p.add_subparsers(dest="cmd", required=True)
    for name in ("download", "tokenize"):
        s = sub.add_parser(name)
        s.add_argument("--sample", default="100BT", choices=fineweb_edu.SAMPLES)
        s.add_argument("--count", type=int, required=True)
    s = sub.add_parser("synthetic")
    s.add_argument("out_dir")
    s.add_argument("--tokens", type=int, required=True)
    s.add_argument("--vocab", type=int, default=32000)
    s.add_argument("--shards", type=int, default=1)
    s.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    if a.cmd == "download":
        paths = fineweb_edu.download(a.sample, a.count)
        print(f"{len(paths)} shards present under {paths[0].parent}")
    elif a.cmd == "tokenize":
        out = Path(__file__).resolve().parents[2] / "data" / "tokenized" / f"fineweb-edu-{a.sample}-mistral32k"
        print("manifest:", prepare(_local_sources(a.sample, a.count, out),
                                   {"repo_id": fineweb_edu.REPO_ID, "revision": fineweb_edu.REVISION,
                                    "sample": a.sample}, out))
    else:
        print("manifest:", synthetic_store(a.out_dir, a.tokens, a.vocab, seed=a.seed, shards=a.shards))


if __name__ == "__main__":
    main()
