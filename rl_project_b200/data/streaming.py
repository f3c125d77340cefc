"""Streaming corpora (capabilities of ``src/forgeline/data/streaming.py``): token shards split over ranks
and loader workers, raw-text globs and HuggingFace streams tokenised on the fly, and a bounded-memory shard
writer.

Two pieces carry the design:

* ``TokenPacker`` -- a growable numpy token buffer with a read cursor.  Documents are appended as arrays
  and every complete ``block_size + 1`` window is emitted as ``(x, y)`` (consecutive windows share one
  token, stride ``block_size``); consumed tokens are compacted away only when the cursor passes half the
  buffer, so packing is linear in the stream length.
* ``ShardWriter`` -- one preallocated shard-sized array; documents of any length are copied into it in
  pieces and full shards flushed to ``<split>_NNNNNN.bin`` (the first one ``val``), then the pieces are
  byte-concatenated into ``train.bin`` / ``val.bin``.
"""

from __future__ import annotations

import glob
import os
import random
import shutil
import time
from pathlib import Path
from typing import Iterable, Iterator, List, Optional, Tuple

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset

from rl_project_b200.core.errors import DatasetError, OptionalDependencyError
from rl_project_b200.observability.logging import get_logger

log = get_logger("data.streaming")

Window = Tuple[torch.Tensor, torch.Tensor]


class TokenPacker:
    """Concatenates token arrays and yields fixed next-token windows."""

    def __init__(self, block_size: int, capacity: int = 1 << 16):
        self.block = block_size
        self.buf = np.empty(max(capacity, 2 * (block_size + 1)), dtype=np.int64)
        self.lo = self.hi = 0  # unread tokens are buf[lo:hi]

    def push(self, ids) -> None:
        ids = np.asarray(ids, dtype=np.int64)
        if self.hi + ids.shape[0] > self.buf.shape[0]:
            live = self.buf[self.lo:self.hi]
            size = max(self.buf.shape[0], 2 * (live.shape[0] + ids.shape[0]))
            fresh = np.empty(size, dtype=np.int64) if size > self.buf.shape[0] else self.buf
            fresh[:live.shape[0]] = live  # overlapping move is safe: numpy copies through a temporary
            self.buf, self.lo, self.hi = fresh, 0, live.shape[0]
        self.buf[self.hi:self.hi + ids.shape[0]] = ids
        self.hi += ids.shape[0]

    def windows(self) -> Iterator[Window]:
        B = self.block
        while self.hi - self.lo >= B + 1:
            w = torch.from_numpy(self.buf[self.lo:self.lo + B + 1].copy())
            self.lo += B
            yield w[:-1], w[1:]


def _keep(text: str, min_chars: int) -> bool:
    return bool(text) and len(text.strip()) >= min_chars


def _doc_ids(tokenizer, text: str, drop_token_zero: bool) -> np.ndarray:
    ids = np.asarray(tokenizer.encode(text), dtype=np.int64)
    return ids[ids != 0] if drop_token_zero else ids


class ShardedTokenDataset(IterableDataset):
    """``(x, y)`` windows from ``shard_*.bin`` files: rank ``r`` of ``world`` owns every ``world``-th shard,
    and loader worker ``w`` every ``num_workers``-th of those.  Shuffled: shard order and window starts are
    drawn from a per-worker seeded generator (``len // block`` random windows per shard); otherwise
    consecutive non-overlapping windows."""

    kind = "pretraining"

    def __init__(self, shard_dir: str | Path, block_size: int, shuffle: bool = True, world_size: int = 1,
                 rank: int = 0, dtype=np.uint16, seed: int = 0, pattern: str = "shard_*.bin"):
        super().__init__()
        self.block_size, self.shuffle, self.dtype, self.seed = block_size, shuffle, np.dtype(dtype), seed
        found = sorted(glob.glob(os.path.join(str(shard_dir), pattern)))
        if not found:
            raise DatasetError(f"No shard files matching {pattern!r} in {shard_dir}")
        self.shard_paths = found[rank::world_size]
        self.total_tokens = sum(os.path.getsize(p) for p in self.shard_paths) // self.dtype.itemsize

    def _starts(self, n: int, rng: random.Random) -> List[int]:
        B = self.block_size
        count = n // B
        if self.shuffle:
            return [rng.randrange(n - B) for _ in range(count)]
        return list(range(0, n - B, B))[:count]

    def __iter__(self) -> Iterator[Window]:
        info = torch.utils.data.get_worker_info()
        wid, nw = (info.id, info.num_workers) if info is not None else (0, 1)
        mine = self.shard_paths[wid::nw]
        rng = random.Random(self.seed + wid)
        if self.shuffle:
            rng.shuffle(mine)
        B = self.block_size
        offsets = np.arange(B + 1)
        for path in mine:
            data = np.memmap(path, dtype=self.dtype, mode="r")
            n = data.shape[0]
            if n <= B:
                continue
            for s in self._starts(n, rng):
                if s + B + 1 > n:  # a window needs its last target token
                    continue
                w = torch.from_numpy(np.asarray(data[s + offsets], dtype=np.int64))
                yield w[:-1], w[1:]


class TextGlobDataset(IterableDataset):
    """Raw text files matching a glob, tokenised line by line and packed into windows."""

    kind = "pretraining"

    def __init__(self, pattern: str, tokenizer, block_size: int, shuffle: bool = True, seed: int = 0):
        super().__init__()
        self.files = sorted(glob.glob(pattern))
        if not self.files:
            raise DatasetError(f"No files matching {pattern!r}")
        self.tokenizer, self.block_size, self.shuffle, self.seed = tokenizer, block_size, shuffle, seed

    def __iter__(self) -> Iterator[Window]:
        order = list(self.files)
        if self.shuffle:
            random.Random(self.seed).shuffle(order)
        packer = TokenPacker(self.block_size)
        for f in order:
            with open(f, "r", errors="ignore") as fh:
                for line in fh:
                    packer.push(self.tokenizer.encode(line))
                    yield from packer.windows()


class HFStreamingDataset(IterableDataset):
    """A streamed HuggingFace dataset (``datasets`` needed), split over ranks and workers, shuffled through a
    10k-example buffer and packed into windows."""

    kind = "pretraining"

    def __init__(self, dataset_name: str, tokenizer, block_size: int, subset: Optional[str] = None,
                 split: str = "train", text_field: str = "text", max_tokens: Optional[int] = None, rank: int = 0,
                 world_size: int = 1, seed: int = 42, min_chars: int = 50):
        super().__init__()
        self.dataset_name, self.subset, self.split, self.text_field = dataset_name, subset, split, text_field
        self.tokenizer, self.block_size, self.max_tokens = tokenizer, block_size, max_tokens
        self.rank, self.world_size, self.seed, self.min_chars = rank, world_size, seed, min_chars

    def _dataset(self):
        try:
            from datasets import load_dataset
        except ImportError as exc:
            raise OptionalDependencyError("datasets is not installed", hint="pip install datasets") from exc
        args = (self.dataset_name, self.subset) if self.subset else (self.dataset_name,)
        ds = load_dataset(*args, streaming=True, split=self.split)
        info = torch.utils.data.get_worker_info()
        for parts, index in ((self.world_size, self.rank),
                             (info.num_workers if info else 1, info.id if info else 0)):
            if parts > 1:
                ds = ds.shard(num_shards=parts, index=index)
        return ds.shuffle(seed=self.seed, buffer_size=10_000)

    def __iter__(self) -> Iterator[Window]:
        texts = (ex.get(self.text_field, "") for ex in self._dataset())
        yield from pack_documents(texts, self.tokenizer, self.block_size, max_tokens=self.max_tokens,
                                  min_chars=self.min_chars)


def pack_documents(texts: Iterable[str], tokenizer, block_size: int, *, max_tokens: Optional[int] = None,
                   min_chars: int = 0, drop_token_zero: bool = False) -> Iterator[Window]:
    """Windows of the concatenated documents (those shorter than ``min_chars`` stripped characters are
    skipped); stops after the document that brings the total past ``max_tokens``."""
    packer = TokenPacker(block_size)
    seen = 0
    for text in texts:
        if not _keep(text, min_chars):
            continue
        ids = _doc_ids(tokenizer, text, drop_token_zero)
        if not ids.shape[0]:
            continue
        packer.push(ids)
        seen += ids.shape[0]
        yield from packer.windows()
        if max_tokens is not None and seen >= max_tokens:
            return


def shard_token_file(input_path: str | Path, output_dir: str | Path, n_shards: int, dtype=np.uint16) -> List[Path]:
    """Split one token file into at most ``n_shards`` near-equal ``shard_NNNN.bin`` files."""
    out_dir = Path(output_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    data = np.memmap(str(input_path), dtype=dtype, mode="r")
    per = -(-data.shape[0] // n_shards)
    paths = []
    for i, a in enumerate(range(0, data.shape[0], per)):
        p = out_dir / f"shard_{i:04d}.bin"
        np.asarray(data[a:a + per]).tofile(p)
        paths.append(p)
    return paths


class ShardWriter:
    """Fixed-size token shards written from a stream of documents (peak memory: one shard)."""

    def __init__(self, output_dir: str | Path, shard_size: int, dtype, first_shard_is_val: bool = True,
                 log_every: int = 1):
        self.dir = Path(output_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.buf = np.empty(shard_size, dtype=dtype)
        self.fill = self.shards = self.flushed = self.docs = 0
        self.first_val, self.log_every = first_shard_is_val, log_every
        self.files: List[Path] = []
        self.t0 = time.time()

    @property
    def pending(self) -> int:
        return self.flushed + self.fill

    def add(self, ids: np.ndarray) -> None:
        self.docs += 1
        ids = ids.astype(self.buf.dtype, copy=False)
        while ids.shape[0]:
            take = min(self.buf.shape[0] - self.fill, ids.shape[0])
            self.buf[self.fill:self.fill + take] = ids[:take]
            self.fill += take
            ids = ids[take:]
            if self.fill == self.buf.shape[0]:
                self.flush()

    def flush(self) -> None:
        if not self.fill:
            return
        split = "val" if self.first_val and self.shards == 0 else "train"
        path = self.dir / f"{split}_{self.shards:06d}.bin"
        self.buf[:self.fill].tofile(path)
        self.files.append(path)
        self.flushed += self.fill
        self.fill = 0
        if self.log_every and self.shards % self.log_every == 0:
            dt = time.time() - self.t0
            log.info("shard_written", index=self.shards, split=split, tokens=self.flushed, docs=self.docs,
                     tok_per_s=round(self.flushed / dt) if dt > 0 else 0)
        self.shards += 1


def write_shards_from_documents(texts: Iterable[str], tokenizer, output_dir: str | Path, *, max_tokens: int,
                                shard_size: int = 10_000_000, dtype=np.uint32, min_chars: int = 50,
                                drop_token_zero: bool = True, first_shard_is_val: bool = True,
                                log_every: int = 1) -> dict:
    """Tokenise ``texts`` into shards, then merge them into ``train.bin`` / ``val.bin``."""
    w = ShardWriter(output_dir, shard_size, dtype, first_shard_is_val, log_every)
    for text in texts:
        if not _keep(text, min_chars):
            continue
        ids = _doc_ids(tokenizer, text, drop_token_zero)
        if ids.shape[0]:
            w.add(ids)
            if w.pending >= max_tokens:
                break
    w.flush()
    merge_shards(output_dir, dtype=dtype)
    return {"total_tokens": w.flushed, "num_shards": w.shards, "docs": w.docs, "files": [str(p) for p in w.files]}


def merge_shards(output_dir: str | Path, dtype=np.uint32, chunk: int = 5_000_000) -> None:
    """Byte-concatenate ``<split>_*.bin`` into ``<split>.bin`` for the train and val splits (``chunk`` ids per
    read)."""
    out_dir = Path(output_dir)
    block = chunk * np.dtype(dtype).itemsize
    for split in ("train", "val"):
        parts = sorted(out_dir.glob(f"{split}_*.bin"))
        if parts:
            with (out_dir / f"{split}.bin").open("wb") as out:
                for part in parts:
                    with part.open("rb") as src:
                        shutil.copyfileobj(src, out, block)


def build_streaming_loader(dataset: IterableDataset, batch_size: int, num_workers: int = 0,
                           pin_memory: bool = False) -> DataLoader:
    return DataLoader(dataset, batch_size=batch_size, num_workers=num_workers,
                      pin_memory=pin_memory and torch.cuda.is_available(), drop_last=True)
