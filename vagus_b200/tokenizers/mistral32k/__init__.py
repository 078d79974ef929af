"""The Mistral-7B-lineage 32k tokenizer (vendored ``tokenizer.json``; hash and
provenance in META.json).  ``encode`` prepends BOS and never appends EOS, so
BOS separates documents in packed streams."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

_DIR = Path(__file__).resolve().parent
_FILE = _DIR / "tokenizer.json"
UNK_ID, BOS_ID, EOS_ID = 0, 1, 2


def load():
    from tokenizers import Tokenizer
    return Tokenizer.from_file(str(_FILE))


def fingerprint() -> str:
    return hashlib.sha256(_FILE.read_bytes()).hexdigest()


def meta() -> dict:
    return json.loads((_DIR / "META.json").read_text())
