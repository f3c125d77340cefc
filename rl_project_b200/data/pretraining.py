"""Pre-tokenised memory-mapped corpora (``src/forgeline/data/pretraining.py``):
``<split>.bin`` of uint16 (or uint32 for vocabularies > 65535 / tiktoken),
random ``(x, y)`` next-token windows drawn with a torch ``Generator``.
Batches are assembled in pinned host memory and copied asynchronously."""

from __future__ import annotations

from pathlib import Path
from typing import Iterator, Optional, Tuple

import numpy as np
import torch

from rl_project_b200.core.errors import DatasetError
from rl_project_b200.data.tokenizers import load_tokenizer_metadata


def detect_token_dtype(data_dir: str | Path) -> np.dtype:
    if not (Path(data_dir) / "meta.pkl").exists():
        return np.dtype(np.uint16)
    meta = load_tokenizer_metadata(data_dir)
    big = int(meta.get("vocab_size", 0)) > 65535 or meta.get("tokenizer_type") == "tiktoken"
    return np.dtype(np.uint32 if big else np.uint16)


class MemmapCorpus:
    kind = "pretraining"

    def __init__(self, data_dir: str | Path, split: str, block_size: int, dtype: Optional[np.dtype] = None):
        self.data_dir = Path(data_dir)
        self.split = split
        self.block_size = block_size
        path = self.data_dir / f"{split}.bin"
        if not path.exists():
            raise DatasetError(f"Token file not found: {path}", hint="Prepare the corpus (`data prepare`) first.")
        self.dtype = dtype or detect_token_dtype(self.data_dir)
        self.data = np.memmap(path, dtype=self.dtype, mode="r")
        if len(self.data) <= block_size + 1:
            raise DatasetError(f"{path} has {len(self.data)} tokens; need more than block_size+1={block_size + 1}")

    def __len__(self) -> int:
        return len(self.data) - self.block_size - 1

    @property
    def n_tokens(self) -> int:
        return int(len(self.data))

    def sample_batch(self, batch_size: int, device: torch.device | str = "cpu",
                     generator: Optional[torch.Generator] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        starts = torch.randint(len(self.data) - self.block_size, (batch_size,), generator=generator).tolist()
        win = np.stack([np.asarray(self.data[s: s + self.block_size + 1], dtype=np.int64) for s in starts])
        t = torch.from_numpy(win)
        dev = torch.device(device)
        if dev.type == "cuda":
            t = t.pin_memory().to(dev, non_blocking=True)
        return t[:, :-1], t[:, 1:]

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        B = self.block_size
        for i in range(0, len(self.data) - B - 1, B):
            w = torch.from_numpy(np.asarray(self.data[i: i + B + 1], dtype=np.int64))
            yield w[:-1], w[1:]


def write_token_file(tokens: np.ndarray, path: str | Path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tokens.tofile(path)
    return path
