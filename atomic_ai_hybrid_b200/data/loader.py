"""Multi-source token dataset and loaders (reference `train_setup.py:639-935`).

Files are ``.npy`` arrays ``[N, ctx]`` of int32 token ids plus an aligned labels
array (either merged ``{prefix}_input_ids.npy``/``{prefix}_labels.npy`` or numbered
shards ``{prefix}_shard_ids_{i}.npy``/``{prefix}_shard_lbls_{i}.npy``), memory
mapped.  The index bookkeeping follows the reference step by step so that the
same files give the same batches:

* per-source fraction (``RandomState(fraction_seed)``), then an optional global
  fraction, then a ``val_split`` hold-out drawn with ``RandomState(42)``;
* modes ``mixed`` (global shuffle per pass with ``RandomState(123)``),
  ``sequential`` (sources one after another) and ``round_robin`` (one source per
  micro-step, source ``s`` shuffled with ``RandomState(1000+s)``); round-robin
  batches carry ``_source_idx``;
* resume skips already-consumed micro-steps without reading from disk.

Each yielded global batch is sliced for the data-parallel rank (rows
``[r*B/W, (r+1)*B/W)``, the reference's batch sharding) and handed over as
pinned host tensors, optionally prefetched by a background thread.
"""
from __future__ import annotations

import glob
import os
import queue
import re
import threading
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np
import torch


def resolve_source_files(output_dir: str, prefix: str) -> List[Tuple[str, str]]:
    merged_ids = os.path.join(output_dir, f"{prefix}_input_ids.npy")
    merged_lbls = os.path.join(output_dir, f"{prefix}_labels.npy")
    if os.path.exists(merged_ids) and os.path.exists(merged_lbls):
        return [(merged_ids, merged_lbls)]
    shard_ids = sorted(glob.glob(os.path.join(output_dir, f"{prefix}_shard_ids_*.npy")),
                       key=lambda p: int(re.search(r"_(\d+)\.npy$", p).group(1)))
    pairs = []
    for ids_path in shard_ids:
        lbls_path = ids_path.replace("_shard_ids_", "_shard_lbls_")
        if os.path.exists(lbls_path):
            pairs.append((ids_path, lbls_path))
    if not pairs:
        raise FileNotFoundError(f"no files for prefix={prefix!r} in {output_dir}: neither {prefix}_input_ids.npy "
                                f"nor {prefix}_shard_ids_*.npy")
    return pairs


def build_manifest(file_pairs: Sequence[Sequence]) -> List[Tuple[str, str, int]]:
    manifest = []
    for entry in file_pairs:
        ids_path, lbls_path = entry[0], entry[1]
        n_rows = np.load(ids_path, mmap_mode="r").shape[0]
        manifest.append((ids_path, lbls_path, int(n_rows)))
    return manifest


class MultiSourceDataset:
    """Index pools of the reference's multi-source loader."""

    def __init__(self, file_pairs, seq_len: int, val_split: float = 0.05, dataset_fraction: float = 1.0,
                 fraction_seed: int = 777):
        norm = []
        for e in file_pairs:
            norm.append((e[0], e[1], float(e[2]) if len(e) == 3 else 1.0))
        self.manifest = build_manifest([(p[0], p[1]) for p in norm])
        sizes = np.array([n for _, _, n in self.manifest])
        self.offsets = np.concatenate([[0], np.cumsum(sizes)])
        ctx = np.load(self.manifest[0][0], mmap_mode="r").shape[1]
        self.context = min(ctx, seq_len)
        self._mmaps: Dict[str, np.ndarray] = {}
        rng = np.random.RandomState(fraction_seed)
        self.per_source: List[np.ndarray] = []
        for s, (_, _, n) in enumerate(self.manifest):
            idx = np.arange(self.offsets[s], self.offsets[s + 1])
            frac = norm[s][2]
            if frac < 1.0:
                keep = max(1, int(len(idx) * frac))
                idx = rng.choice(idx, size=keep, replace=False)
                idx.sort()
            self.per_source.append(idx)
        all_idx = np.concatenate(self.per_source)
        if dataset_fraction < 1.0:
            frng = np.random.RandomState(fraction_seed)
            all_idx = frng.choice(all_idx, size=int(len(all_idx) * dataset_fraction), replace=False)
            all_idx.sort()
        pool = len(all_idx)
        val_size = int(pool * val_split)
        split = np.random.RandomState(42)
        sh = np.copy(all_idx)
        split.shuffle(sh)
        self.train_pool = sh[:pool - val_size]
        self.val_pool = sh[pool - val_size:]
        val_set = set(self.val_pool.tolist())
        self.train_by_source = [np.array([i for i in src if i not in val_set], dtype=np.int64)
                                for src in self.per_source]

    def _mmap(self, path):
        a = self._mmaps.get(path)
        if a is None:
            a = np.load(path, mmap_mode="r")
            self._mmaps[path] = a
        return a

    def gather(self, idx: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
        shard = np.searchsorted(self.offsets, idx, side="right") - 1
        ids = np.empty((len(idx), self.context), dtype=np.int32)
        lbl = np.empty((len(idx), self.context), dtype=np.int32)
        for s in np.unique(shard):
            m = shard == s
            local = idx[m] - self.offsets[s]
            ip, lp, _ = self.manifest[s]
            ids[m] = self._mmap(ip)[local][:, :self.context]
            lbl[m] = self._mmap(lp)[local][:, :self.context]
        return ids, lbl

    # ------------------------------------------------------------ index streams
    def mixed_indices(self, batch: int, train: bool = True, skip: int = 0) -> Iterator[np.ndarray]:
        idx = np.copy(self.train_pool if train else self.val_pool)
        rng = np.random.RandomState(123)
        first = True
        while True:
            if train:
                rng.shuffle(idx)
            n = len(idx) // batch
            start = (skip % max(n, 1)) if (first and train) else 0
            first = False
            for step in range(start, n):
                yield idx[step * batch:(step + 1) * batch]
            if not train:
                return

    def sequential_indices(self, batch: int, skip: int = 0) -> Iterator[Tuple[int, np.ndarray]]:
        rng = np.random.RandomState(123)
        remaining = skip
        first = True
        while True:
            for s, src in enumerate(self.train_by_source):
                idx = np.copy(src)
                rng.shuffle(idx)
                n = len(idx) // batch
                start = 0
                if first and remaining > 0:
                    start = min(remaining, n)
                    remaining -= start
                for step in range(start, n):
                    yield s, idx[step * batch:(step + 1) * batch]
            first = False

    def round_robin_indices(self, batch: int, skip: int = 0) -> Iterator[Tuple[int, np.ndarray]]:
        def src_stream(src, seed):
            rng = np.random.RandomState(seed)
            idx = np.copy(src)
            while True:
                rng.shuffle(idx)
                for step in range(len(idx) // batch):
                    yield idx[step * batch:(step + 1) * batch]

        gens = [src_stream(self.train_by_source[s], 1000 + s) for s in range(len(self.train_by_source))]
        i = 0
        while True:
            s = i % len(gens)
            b = next(gens[s])
            i += 1
            if i <= skip:
                continue
            yield s, b


def _to_batch(ids: np.ndarray, lbl: np.ndarray, rank: int, world: int, pin: bool) -> Dict[str, torch.Tensor]:
    per = ids.shape[0] // world
    a = torch.from_numpy(np.ascontiguousarray(ids[rank * per:(rank + 1) * per])).long()
    b = torch.from_numpy(np.ascontiguousarray(lbl[rank * per:(rank + 1) * per])).long()
    if pin and torch.cuda.is_available():
        a, b = a.pin_memory(), b.pin_memory()
    return {"input_ids": a, "labels": b}


def dataloader_multi_source(file_pairs, batch_size: int, seq_len: int, val_split: float = 0.05,
                            dataset_fraction: float = 1.0, fraction_seed: int = 777, skip_batches: int = 0,
                            mode: str = "mixed", rank: int = 0, world: int = 1, pin: bool = True):
    """Returns ``(train_iter, val_factory, train_steps_per_epoch, val_steps)`` like the
    reference; batches are the rank's slice of the global ``batch_size`` rows."""
    if batch_size % world:
        raise ValueError(f"batch_size={batch_size} must be divisible by world={world}")
    ds = MultiSourceDataset(file_pairs, seq_len, val_split, dataset_fraction, fraction_seed)

    def train_iter():
        if mode == "mixed":
            for idx in ds.mixed_indices(batch_size, True, skip_batches):
                yield _to_batch(*ds.gather(idx), rank, world, pin)
        elif mode in ("sequential", "round_robin"):
            gen = ds.sequential_indices(batch_size, skip_batches) if mode == "sequential" else \
                ds.round_robin_indices(batch_size, skip_batches)
            for s, idx in gen:
                b = _to_batch(*ds.gather(idx), rank, world, pin)
                b["_source_idx"] = s
                yield b
        else:
            raise ValueError(f"unknown mode={mode!r}: expected 'mixed', 'sequential' or 'round_robin'")

    def val_iter():
        for idx in ds.mixed_indices(batch_size, False):
            yield _to_batch(*ds.gather(idx), rank, world, pin)

    return train_iter(), val_iter, len(ds.train_pool) // batch_size, len(ds.val_pool) // batch_size


class Prefetcher:
    """Runs a batch iterator in a background thread (``depth`` batches ahead)."""

    def __init__(self, it: Iterator, depth: int = 4):
        self.q: "queue.Queue" = queue.Queue(maxsize=depth)
        self._done = object()

        def work():
            try:
                for b in it:
                    self.q.put(b)
            finally:
                self.q.put(self._done)

        self.t = threading.Thread(target=work, daemon=True)
        self.t.start()

    def __iter__(self):
        return self

    def __next__(self):
        b = self.q.get()
        if b is self._done:
            raise StopIteration
        return b


def synthetic_batches(vocab: int, batch: int, seq_len: int, seed: int = 0, rank: int = 0,
                      world: int = 1) -> Iterator[Dict[str, torch.Tensor]]:
    """Uniform random token ids (next-token labels), the benchmark's synthetic data."""
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    while True:
        ids = torch.randint(0, vocab, (batch // world, seq_len + 1), generator=g)
        yield {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}


_ = Optional
