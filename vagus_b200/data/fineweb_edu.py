"""FineWeb-Edu acquisition: pinned-revision download of raw parquet shards
(name-sorted prefixes only, idempotent).  Network access is only needed
here; tokenisation and training read local files.

Parity: reference ``infra/dataset/fineweb_edu.py:7-74``.
"""

from __future__ import annotations

from pathlib import Path

REPO_ID = "HuggingFaceFW/fineweb-edu"
REVISION = "87f09149ef4734204d70ed1d046ddc9ca3f2b8f9"
SAMPLES = ("10BT", "100BT", "350BT")


def default_dest() -> Path:
    return Path(__file__).resolve().parents[2] / "data" / "fineweb-edu"


def download(sample: str = "10BT", file_count: int | None = None, dest=None) -> list[Path]:
    assert sample in SAMPLES
    dest = Path(dest) if dest is not None else default_dest()
    have = sorted((dest / "sample" / sample).glob("*.parquet"))
    if file_count is not None and len(have) >= file_count:
        return have[:file_count]
    from huggingface_hub import HfApi, snapshot_download   # network; prep machines only
    names = sorted(e.path for e in HfApi().list_repo_tree(REPO_ID, f"sample/{sample}", repo_type="dataset",
                                                          revision=REVISION) if e.path.endswith(".parquet"))
    if file_count is not None:
        if file_count > len(names):
            raise ValueError(f"sample/{sample} has only {len(names)} shards.")
        names = names[:file_count]
    snapshot_download(REPO_ID, repo_type="dataset", revision=REVISION, local_dir=dest, allow_patterns=names)
    return [dest / n for n in names]
