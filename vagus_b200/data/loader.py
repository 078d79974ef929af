"""Training-side reading of ``vagus-tokens-v1`` datasets.

``TokenStore``   manifest-backed view of a tokenised dataset: per shard a
                 uint16 ``.npy`` token stream (per-document BOS, no EOS) and a
                 uint64 ``.idx.npy`` of document offsets.  Windows are read
                 with ``os.pread`` (the GIL is released during the disk wait);
                 memmaps stay for document addressing.
``WindowLoader`` uniform non-overlapping windows of context_len + 1 tokens,
                 reshuffled per epoch by ``default_rng((seed, epoch))``, ranks
                 taking interleaved slices of the global order (global batch
                 g = batch_in_epoch * world + rank), exactly resumable from
                 (epoch, batch_in_epoch) with a fingerprint of the order-defining
                 parameters.  A background thread prefetches batches into
                 pinned host memory so the host -> device copy can overlap the
                 step.  The batch sequence is a pure function of (seed, epoch,
                 rank, batch index) and identical with or without prefetch.

Parity: reference ``infra/dataset/loader.py:31-246`` (format, window policy,
order, state dict and fingerprint are the same).
"""

from __future__ import annotations

import json
import os
import queue
import threading
from pathlib import Path

import numpy as np
import torch

FORMAT = "vagus-tokens-v1"


class TokenStore:
    def __init__(self, manifest_dir: str | Path, shards: list[str] | None = None):
        self.dir = Path(manifest_dir)
        self.manifest = json.loads((self.dir / "manifest.json").read_text())
        assert self.manifest["format"] == FORMAT
        assert self.manifest["dtype"] == "uint16"
        entries = sorted(self.manifest["shards"], key=lambda s: s["source"])
        if shards is not None:
            by_name = {e["file"]: e for e in entries}
            entries = [by_name[name] for name in shards]
        self.entries = entries
        self.tokens: list[np.ndarray] = [np.load(self.dir / e["file"], mmap_mode="r") for e in entries]
        for arr, e in zip(self.tokens, entries):
            assert arr.dtype == np.uint16 and len(arr) == e["tokens"]
        self.shard_tokens = [len(a) for a in self.tokens]
        self.total_tokens = sum(self.shard_tokens)
        self.vocab_size = self.manifest["tokenizer"]["vocab_size"]
        self._fds = [os.open(str(self.dir / e["file"]), os.O_RDONLY) for e in entries]
        self._data_off = [int(a.offset) for a in self.tokens]
        self._idx: list[np.ndarray | None] = [None] * len(entries)

    def read_window(self, shard: int, start: int, count: int) -> np.ndarray:
        buf = os.pread(self._fds[shard], count * 2, self._data_off[shard] + start * 2)
        assert len(buf) == count * 2, f"short read: shard {shard} @ {start}+{count}"
        return np.frombuffer(buf, dtype=np.uint16)

    def doc_offsets(self, shard: int) -> np.ndarray:
        idx = self._idx[shard]
        if idx is None:
            idx = np.load(self.dir / self.entries[shard]["idx"], mmap_mode="r")
            self._idx[shard] = idx
        return idx

    def doc(self, shard: int, i: int) -> np.ndarray:
        off = self.doc_offsets(shard)
        return self.tokens[shard][int(off[i]):int(off[i + 1])]

    def __del__(self):
        for fd in getattr(self, "_fds", []):
            try:
                os.close(fd)
            except OSError:
                pass


class WindowLoader:
    def __init__(self, store: TokenStore, context_len: int, batch_size: int, *, seed: int = 0, rank: int = 0,
                 world_size: int = 1, shuffle: bool = True, prefetch: int = 4, pin_memory: bool = False):
        assert context_len > 0 and batch_size > 0
        assert 0 <= rank < world_size
        assert prefetch >= 0
        self.store = store
        self.context_len = context_len
        self.batch_size = batch_size
        self.seed = seed
        self.rank = rank
        self.world_size = world_size
        self.shuffle = shuffle
        self.prefetch = prefetch
        self.pin_memory = pin_memory and torch.cuda.is_available()
        # window k of a shard starts at k * context_len and spans context_len + 1 tokens
        per_shard = [(n - 1) // context_len for n in store.shard_tokens]
        bases = np.cumsum([0] + store.shard_tokens[:-1])
        self._starts = (np.concatenate([b + np.arange(w, dtype=np.int64) * context_len
                                        for w, b in zip(per_shard, bases)])
                        if per_shard else np.zeros(0, dtype=np.int64))
        self._shard_base = np.cumsum([0] + store.shard_tokens)
        self.window_count = len(self._starts)
        self.batches_per_epoch = self.window_count // (world_size * batch_size)
        assert self.batches_per_epoch > 0, "fewer windows than one global batch"
        self.tokens_per_batch = batch_size * context_len
        self.epoch = 0
        self.batch_in_epoch = 0

    def _epoch_order(self, epoch: int) -> np.ndarray:
        if not self.shuffle:
            return self._starts
        return self._starts[np.random.default_rng((self.seed, epoch)).permutation(self.window_count)]

    def _fingerprint(self) -> tuple:
        return (self.window_count, self.context_len, self.batch_size, self.seed, self.world_size, self.shuffle)

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "batch_in_epoch": self.batch_in_epoch, "fingerprint": self._fingerprint()}

    def load_state_dict(self, state: dict) -> None:
        if tuple(state["fingerprint"]) != self._fingerprint():
            raise ValueError("loader state was produced under a different data order (fingerprint mismatch)")
        self.epoch = state["epoch"]
        self.batch_in_epoch = state["batch_in_epoch"]

    def _gather(self, flat_starts: np.ndarray):
        L = self.context_len
        out = torch.empty((len(flat_starts), L + 1), dtype=torch.int64, pin_memory=self.pin_memory)
        arr = out.numpy()
        for row, flat in enumerate(flat_starts):
            s = int(np.searchsorted(self._shard_base, flat, side="right")) - 1
            arr[row] = self.store.read_window(s, int(flat - self._shard_base[s]), L + 1)
        return out[:, :-1], out[:, 1:]

    def _produce(self, epoch: int, batch_in_epoch: int):
        B, W, R = self.batch_size, self.world_size, self.rank
        while True:
            order = self._epoch_order(epoch)
            while batch_in_epoch < self.batches_per_epoch:
                g = batch_in_epoch * W + R
                x, y = self._gather(order[g * B:(g + 1) * B])
                yield epoch, batch_in_epoch, x, y
                batch_in_epoch += 1
            epoch += 1
            batch_in_epoch = 0

    def __iter__(self):
        src = self._produce(self.epoch, self.batch_in_epoch)
        if self.prefetch == 0:
            for epoch, b, x, y in src:
                self.epoch, self.batch_in_epoch = epoch, b + 1
                yield x, y
            return
        q: queue.Queue = queue.Queue(maxsize=self.prefetch)
        stop = threading.Event()

        def reader():
            try:
                for item in src:
                    while not stop.is_set():
                        try:
                            q.put(item, timeout=1.0)
                            break
                        except queue.Full:
                            pass
                    else:
                        return
            except BaseException as e:  # surfaced in the consumer
                q.put(e)

        threading.Thread(target=reader, daemon=True, name="WindowLoader-prefetch").start()
        try:
            while True:
                item = q.get()
                if isinstance(item, BaseException):
                    raise item
                epoch, b, x, y = item
                self.epoch, self.batch_in_epoch = epoch, b + 1
                yield x, y
        finally:
            stop.set()
