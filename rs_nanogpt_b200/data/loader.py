"""Pretraining data pipeline (rs-nanogpt src/data/parquet.rs, src/data/loader.rs).

* Shards: sorted ``*.parquet`` files of a directory; the last one is the
  validation split, the rest train (at least two are required).
* Documents: the non-null ``text`` column, strided by rank *before*
  tokenization (document ``i`` belongs to rank ``i % world``); each non-empty
  document is encoded and prefixed with BOS.
* Packing: best-fit crop packing into rows of T+1 tokens with a pool of 1000
  documents (C++ ``CropPacker``); the source cycles when exhausted.
* Batches: ``inputs = row[:T]`` (int64 ids) and ``targets = row[1:]``.

Unlike the reference, which tokenizes and packs synchronously on the training
thread, a background producer thread (parquet reading through Arrow, C++
tokenization on a thread pool with the GIL released, C++ packing) fills a
queue of pinned host batches ahead of the trainer; ``next_batch`` only copies
one pinned batch to the device asynchronously.
"""
import os
import queue
import threading
from dataclasses import dataclass
from typing import Iterator, List, Optional

import numpy as np
import torch

from .. import _host
from ..tokenizer import BpeTokenizer

DEFAULT_BUFFER_SIZE = 1000


def list_shards(directory: str) -> List[str]:
    if not os.path.isdir(directory):
        raise NotADirectoryError(f"{directory} is not a directory")
    return sorted(os.path.join(directory, f) for f in os.listdir(directory) if f.endswith(".parquet"))


def shards_for_split(all_shards: List[str], split: str) -> List[str]:
    if len(all_shards) < 2:
        raise ValueError(f"need at least 2 shards to form train/val splits, found {len(all_shards)}")
    return all_shards[:-1] if split == "train" else all_shards[-1:]


def iter_texts(shards: List[str], rank: int = 0, world: int = 1, batch_docs: int = 256) -> Iterator[List[str]]:
    """Yield lists of this rank's document texts (global index % world == rank)."""
    import pyarrow.parquet as pq

    if not (world >= 1 and 0 <= rank < world):
        raise ValueError(f"invalid rank {rank} / world {world}")
    index = 0
    out: List[str] = []
    for path in shards:
        pf = pq.ParquetFile(path)
        for batch in pf.iter_batches(columns=["text"]):
            for val in batch.column(0).to_pylist():
                if val is None:
                    continue
                if index % world == rank:
                    out.append(val)
                index += 1
                if len(out) >= batch_docs:
                    yield out
                    out = []
    if out:
        yield out


def split_rows(rows: np.ndarray, batch: int, seq: int):
    rows = rows.reshape(batch, seq + 1)
    return rows[:, :seq].astype(np.int64), rows[:, 1:].astype(np.int64)


@dataclass
class Batch:
    inputs: torch.Tensor   # (B, T) int64
    targets: torch.Tensor  # (B, T) int64, -1 = ignore


class BatchPacker:
    """Synchronous packer: the exact batch sequence of the reference loader."""

    def __init__(self, shards: List[str], tokenizer: BpeTokenizer, batch: int, seq: int,
                 rank: int = 0, world: int = 1, buffer_size: int = DEFAULT_BUFFER_SIZE, threads: int = 0):
        self.shards, self.tok, self.batch, self.seq = shards, tokenizer, batch, seq
        self.rank, self.world, self.threads = rank, world, threads
        self.packer = _host.CropPacker(batch, seq, buffer_size)
        self._texts = iter_texts(shards, rank, world)

    def next_rows(self) -> np.ndarray:
        while not self.packer.step():
            try:
                texts = next(self._texts)
            except StopIteration:
                self.packer.end_pass()  # raises on a pass without documents
                self._texts = iter_texts(self.shards, self.rank, self.world)
                continue
            self.packer.encode_and_push(self.tok.core, texts, self.threads)
        return self.packer.take_rows()

    def next_arrays(self):
        return split_rows(self.next_rows(), self.batch, self.seq)


class DataLoader:
    """Prefetching loader: a producer thread keeps `prefetch` pinned batches ready."""

    def __init__(self, directory: str, split: str, tokenizer: BpeTokenizer, batch: int, seq: int,
                 rank: int = 0, world: int = 1, buffer_size: int = DEFAULT_BUFFER_SIZE, prefetch: int = 4,
                 device: Optional[torch.device] = None):
        shards = shards_for_split(list_shards(directory), split)
        self.packer = BatchPacker(shards, tokenizer, batch, seq, rank, world, buffer_size)
        self.batch, self.seq = batch, seq
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.pin = self.device.type == "cuda"
        self._q: "queue.Queue" = queue.Queue(maxsize=max(1, prefetch))
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._produce, name="nanogpt-data", daemon=True)
        self._thread.start()

    def _produce(self):
        try:
            while not self._stop.is_set():
                x, y = self.packer.next_arrays()
                xt, yt = torch.from_numpy(x), torch.from_numpy(y)
                if self.pin:
                    xt, yt = xt.pin_memory(), yt.pin_memory()
                while not self._stop.is_set():
                    try:
                        self._q.put((xt, yt), timeout=0.5)
                        break
                    except queue.Full:
                        continue
        except BaseException as e:  # surfaced to the consumer
            self._q.put(e)

    def next_host(self):
        item = self._q.get()
        if isinstance(item, BaseException):
            raise item
        return item

    def next_batch(self) -> Batch:
        x, y = self.next_host()
        nb = self.pin
        return Batch(x.to(self.device, non_blocking=nb), y.to(self.device, non_blocking=nb))

    def take_batches(self, n: int) -> List[Batch]:
        return [self.next_batch() for _ in range(n)]

    def close(self):
        self._stop.set()
