"""Training-side reading of ``vagus-tokens-v1`` datasets.

``TokenStore``   manifest-backed view of a tokenised dataset: per shard a
                 uint16 ``.npy`` token stream (per-document BOS, no EOS) and a
                 uint64 ``.idx.npy`` of document offsets.  Windows are read
                 with ``os.pread`` (the GIL is released during the disk wait);
                 memmaps stay for document addressing.
``WindowOrder``  the data-order contract: non-overlapping windows of
                 context_len + 1 tokens, permuted per epoch by
                 ``default_rng((seed, epoch))``, global batch g = b * world +
                 rank, and the fingerprint of everything the order depends on.
``WindowLoader`` one rank's batches in that order, read by a prefetch thread
                 into pinned host memory, exactly resumable from (epoch, batch
                 in epoch); the sequence is the same with or without prefetch.

Parity: reference ``infra/dataset/loader.py`` (store format, window policy,
order, state dict and fingerprint are the same, so a run resumes and pairs
across frameworks on identical data).
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


class WindowOrder:
    """Which windows a rank reads, batch by batch: the data-order contract.

    Window w of a shard spans tokens [w L, w L + L + 1) (L = context_len).
    Epoch e visits all windows in ``default_rng((seed, e)).permutation``
    order (unshuffled: store order); global batch g of an epoch is the
    ``batch_size`` windows at positions [g B, g B + B) of that order, and rank
    R of W takes global batches g = b W + R for its b-th batch.  The
    fingerprint names every parameter the order depends on, so a resume
    under a different one is refused."""

    def __init__(self, store: "TokenStore", context_len: int, batch_size: int, seed: int, rank: int, world: int,
                 shuffle: bool):
        self.L, self.B, self.seed, self.rank, self.world, self.shuffle = \
            context_len, batch_size, seed, rank, world, shuffle
        counts = [(n - 1) // context_len for n in store.shard_tokens]
        first = np.cumsum([0] + store.shard_tokens[:-1])
        # flat start (in the concatenated store) of every window, store order
        self.starts = (np.concatenate([f + context_len * np.arange(c, dtype=np.int64) for c, f in zip(counts, first)])
                       if counts else np.zeros(0, dtype=np.int64))
        self.shard_edges = np.cumsum([0] + store.shard_tokens)
        self.windows = len(self.starts)
        self.batches_per_epoch = self.windows // (world * batch_size)
        self._cached: tuple[int, np.ndarray] | None = None

    def fingerprint(self) -> tuple:
        return (self.windows, self.L, self.B, self.seed, self.world, self.shuffle)

    def epoch_starts(self, epoch: int) -> np.ndarray:
        if not self.shuffle:
            return self.starts
        if self._cached is None or self._cached[0] != epoch:
            perm = np.random.default_rng((self.seed, epoch)).permutation(self.windows)
            self._cached = (epoch, self.starts[perm])
        return self._cached[1]

    def batch(self, epoch: int, b: int) -> tuple[np.ndarray, np.ndarray]:
        """(shard, offset in shard) of the windows of this rank's batch b."""
        g = b * self.world + self.rank
        flat = self.epoch_starts(epoch)[g * self.B:(g + 1) * self.B]
        shard = np.searchsorted(self.shard_edges, flat, side="right") - 1
        return shard, flat - self.shard_edges[shard]


class _Prefetcher:
    """A daemon thread running ``produce`` ahead of the consumer into a
    bounded queue; an exception in the thread is raised in the consumer, and
    ``close`` stops the thread at its next hand-off."""

    def __init__(self, produce, depth: int):
        self.q: queue.Queue = queue.Queue(maxsize=depth)
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._run, args=(produce,), daemon=True, name="WindowLoader-prefetch")
        self.thread.start()

    def _run(self, produce) -> None:
        try:
            for item in produce:
                while not self.stop.is_set():
                    try:
                        self.q.put(item, timeout=1.0)
                        break
                    except queue.Full:
                        continue
                if self.stop.is_set():
                    return
        except BaseException as e:  # noqa: BLE001 -- handed to the consumer
            self.q.put(e)

    def __iter__(self):
        while True:
            item = self.q.get()
            if isinstance(item, BaseException):
                raise item
            yield item

    def close(self) -> None:
        self.stop.set()


class WindowLoader:
    """Batches (x, y) of int64 token windows (B, L) for one rank, in the
    order of ``WindowOrder``, from a background prefetcher into pinned host
    memory (``pin_memory`` on CUDA hosts) so the copy to the device can
    overlap the step.  ``state_dict`` / ``load_state_dict`` resume exactly at
    (epoch, batch in epoch)."""

    def __init__(self, store: TokenStore, context_len: int, batch_size: int, *, seed: int = 0, rank: int = 0,
                 world_size: int = 1, shuffle: bool = True, prefetch: int = 4, pin_memory: bool = False):
        if context_len <= 0 or batch_size <= 0 or not 0 <= rank < world_size or prefetch < 0:
            raise ValueError("WindowLoader: bad context_len / batch_size / rank / prefetch")
        self.store = store
        self.context_len, self.batch_size, self.seed = context_len, batch_size, seed
        self.rank, self.world_size, self.shuffle, self.prefetch = rank, world_size, shuffle, prefetch
        self.pin_memory = pin_memory and torch.cuda.is_available()
        self.order = WindowOrder(store, context_len, batch_size, seed, rank, world_size, shuffle)
        self.window_count = self.order.windows
        self.batches_per_epoch = self.order.batches_per_epoch
        if self.batches_per_epoch <= 0:
            raise ValueError(f"the store holds {self.window_count} windows of {context_len + 1} tokens: fewer than "
                             f"one global batch ({world_size} x {batch_size})")
        self.tokens_per_batch = batch_size * context_len
        self.epoch = 0
        self.batch_in_epoch = 0

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "batch_in_epoch": self.batch_in_epoch, "fingerprint": self.order.fingerprint()}

    def load_state_dict(self, state: dict) -> None:
        if tuple(state["fingerprint"]) != self.order.fingerprint():
            raise ValueError(f"this checkpoint's data order {tuple(state['fingerprint'])} differs from the loader's "
                             f"{self.order.fingerprint()} (windows, context, batch, seed, world, shuffle)")
        self.epoch = state["epoch"]
        self.batch_in_epoch = state["batch_in_epoch"]

    def _read(self, epoch: int, b: int):
        shard, off = self.order.batch(epoch, b)
        L = self.context_len
        buf = torch.empty((self.batch_size, L + 1), dtype=torch.int64, pin_memory=self.pin_memory)
        rows = buf.numpy()
        for i in range(self.batch_size):
            rows[i] = self.store.read_window(int(shard[i]), int(off[i]), L + 1)
        return epoch, b, buf[:, :-1], buf[:, 1:]

    def _batches(self, epoch: int, b: int):
        while True:
            while b < self.batches_per_epoch:
                yield self._read(epoch, b)
                b += 1
            epoch, b = epoch + 1, 0

    def __iter__(self):
        src = self._batches(self.epoch, self.batch_in_epoch)
        pre = _Prefetcher(src, self.prefetch) if self.prefetch else None
        try:
            for epoch, b, x, y in (pre if pre is not None else src):
                self.epoch, self.batch_in_epoch = epoch, b + 1      # the position after this batch
                yield x, y
        finally:
            if pre is not None:
                pre.close()
