"""Streaming corpora (``src/forgeline/data/streaming.py:26-246`` behaviour):
rank/worker-sharded token shards, raw-text globs, HuggingFace streams, a
constant-memory document packer and a fixed-buffer shard writer."""

from __future__ import annotations

import glob
import math
import os
import random
import time
from pathlib import Path
from typing import Iterable, Iterator, List, Optional, Tuple

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset

from rl_project_b200.core.errors import DatasetError, OptionalDependencyError
from rl_project_b200.observability.logging import get_logger

log = get_logger("data.streaming")


def _window(buf: List[int], block: int) -> Tuple[torch.Tensor, torch.Tensor]:
    chunk = torch.tensor(buf[: block + 1], dtype=torch.long)
    return chunk[:-1], chunk[1:]


class ShardedTokenDataset(IterableDataset):
    kind = "pretraining"

    def __init__(self, shard_dir: str | Path, block_size: int, shuffle: bool = True, world_size: int = 1,
                 rank: int = 0, dtype=np.uint16, seed: int = 0, pattern: str = "shard_*.bin"):
        super().__init__()
        self.block_size, self.shuffle, self.dtype, self.seed = block_size, shuffle, dtype, seed
        paths = sorted(glob.glob(os.path.join(str(shard_dir), pattern)))
        if not paths:
            raise DatasetError(f"No shard files matching {pattern!r} in {shard_dir}")
        self.shard_paths = paths[rank::world_size]
        self.total_tokens = sum(os.path.getsize(p) // np.dtype(dtype).itemsize for p in self.shard_paths)

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        info = torch.utils.data.get_worker_info()
        shards = list(self.shard_paths)
        if info is not None:
            shards = shards[info.id::info.num_workers]
        rng = random.Random(self.seed + (info.id if info else 0))
        if self.shuffle:
            rng.shuffle(shards)
        B = self.block_size
        for path in shards:
            data = np.memmap(path, dtype=self.dtype, mode="r")
            n = len(data)
            if n <= B:
                continue
            count = n // B
            starts = ([rng.randrange(0, n - B) for _ in range(count)] if self.shuffle
                      else list(range(0, n - B, B))[:count])
            for s in starts:
                w = torch.from_numpy(np.asarray(data[s: s + B + 1], dtype=np.int64))
                if w.numel() == B + 1:
                    yield w[:-1], w[1:]


class TextGlobDataset(IterableDataset):
    kind = "pretraining"

    def __init__(self, pattern: str, tokenizer, block_size: int, shuffle: bool = True, seed: int = 0):
        super().__init__()
        self.files = sorted(glob.glob(pattern))
        if not self.files:
            raise DatasetError(f"No files matching {pattern!r}")
        self.tokenizer, self.block_size, self.shuffle, self.seed = tokenizer, block_size, shuffle, seed

    def __iter__(self):
        files = list(self.files)
        if self.shuffle:
            random.Random(self.seed).shuffle(files)
        buf: List[int] = []
        for f in files:
            with open(f, "r", errors="ignore") as fh:
                for line in fh:
                    buf.extend(self.tokenizer.encode(line))
                    while len(buf) >= self.block_size + 1:
                        yield _window(buf, self.block_size)
                        buf = buf[self.block_size:]


class HFStreamingDataset(IterableDataset):
    kind = "pretraining"

    def __init__(self, dataset_name: str, tokenizer, block_size: int, subset: Optional[str] = None,
                 split: str = "train", text_field: str = "text", max_tokens: Optional[int] = None, rank: int = 0,
                 world_size: int = 1, seed: int = 42, min_chars: int = 50):
        super().__init__()
        self.dataset_name, self.subset, self.split = dataset_name, subset, split
        self.tokenizer, self.block_size, self.text_field = tokenizer, block_size, text_field
        self.max_tokens, self.rank, self.world_size, self.seed, self.min_chars = max_tokens, rank, world_size, seed, min_chars

    def _dataset(self):
        try:
            from datasets import load_dataset
        except ImportError as exc:
            raise OptionalDependencyError("datasets is not installed", hint="pip install datasets") from exc
        ds = (load_dataset(self.dataset_name, self.subset, streaming=True, split=self.split) if self.subset
              else load_dataset(self.dataset_name, streaming=True, split=self.split))
        if self.world_size > 1:
            ds = ds.shard(num_shards=self.world_size, index=self.rank)
        info = torch.utils.data.get_worker_info()
        if info is not None:
            ds = ds.shard(num_shards=info.num_workers, index=info.id)
        return ds.shuffle(seed=self.seed, buffer_size=10_000)

    def __iter__(self):
        yield from pack_documents((ex.get(self.text_field, "") for ex in self._dataset()), self.tokenizer,
                                  self.block_size, max_tokens=self.max_tokens, min_chars=self.min_chars)


def pack_documents(texts: Iterable[str], tokenizer, block_size: int, *, max_tokens: Optional[int] = None,
                   min_chars: int = 0, drop_token_zero: bool = False):
    buf: List[int] = []
    total = 0
    for text in texts:
        if not text or len(text.strip()) < min_chars:
            continue
        ids = tokenizer.encode(text)
        if drop_token_zero:
            ids = [t for t in ids if t != 0]
        if not ids:
            continue
        buf.extend(ids)
        total += len(ids)
        while len(buf) >= block_size + 1:
            yield _window(buf, block_size)
            buf = buf[block_size:]
        if max_tokens is not None and total >= max_tokens:
            break


def shard_token_file(input_path: str | Path, output_dir: str | Path, n_shards: int, dtype=np.uint16) -> List[Path]:
    out_dir = Path(output_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    data = np.memmap(str(input_path), dtype=dtype, mode="r")
    per = math.ceil(len(data) / n_shards)
    out = []
    for i in range(n_shards):
        a, b = i * per, min((i + 1) * per, len(data))
        if a >= b:
            break
        p = out_dir / f"shard_{i:04d}.bin"
        np.asarray(data[a:b], dtype=dtype).tofile(p)
        out.append(p)
    return out


def write_shards_from_documents(texts: Iterable[str], tokenizer, output_dir: str | Path, *, max_tokens: int,
                                shard_size: int = 10_000_000, dtype=np.uint32, min_chars: int = 50,
                                drop_token_zero: bool = True, first_shard_is_val: bool = True,
                                log_every: int = 1) -> dict:
    out_dir = Path(output_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    buf = np.empty((shard_size,), dtype=dtype)
    fill = index = total = docs = 0
    written: List[Path] = []
    t0 = time.time()

    def flush(n: int) -> None:
        nonlocal index, total
        split = "val" if (first_shard_is_val and index == 0) else "train"
        p = out_dir / f"{split}_{index:06d}.bin"
        buf[:n].tofile(p)
        written.append(p)
        total += n
        if log_every and index % log_every == 0:
            dt = time.time() - t0
            log.info("shard_written", index=index, split=split, tokens=total, docs=docs,
                     tok_per_s=round(total / dt) if dt > 0 else 0)
        index += 1

    for text in texts:
        if not text or len(text.strip()) < min_chars:
            continue
        ids = tokenizer.encode(text)
        if drop_token_zero:
            ids = [t for t in ids if t != 0]
        if not ids:
            continue
        toks = np.asarray(ids, dtype=dtype)
        docs += 1
        pos = 0
        while pos < len(toks):
            take = min(shard_size - fill, len(toks) - pos)
            buf[fill: fill + take] = toks[pos: pos + take]
            fill += take
            pos += take
            if fill == shard_size:
                flush(shard_size)
                fill = 0
        if total + fill >= max_tokens:
            break
    if fill:
        flush(fill)
    merge_shards(out_dir, dtype=dtype)
    return {"total_tokens": total, "num_shards": index, "docs": docs, "files": [str(p) for p in written]}


def merge_shards(output_dir: str | Path, dtype=np.uint32, chunk: int = 5_000_000) -> None:
    out_dir = Path(output_dir)
    for split in ("train", "val"):
        files = sorted(out_dir.glob(f"{split}_*.bin"))
        if not files:
            continue
        with (out_dir / f"{split}.bin").open("wb") as out:
            for fp in files:
                data = np.fromfile(fp, dtype=dtype)
                for i in range(0, len(data), chunk):
                    data[i: i + chunk].tofile(out)


def build_streaming_loader(dataset: IterableDataset, batch_size: int, num_workers: int = 0,
                           pin_memory: bool = False) -> DataLoader:
    return DataLoader(dataset, batch_size=batch_size, num_workers=num_workers,
                      pin_memory=pin_memory and torch.cuda.is_available(), drop_last=True)
