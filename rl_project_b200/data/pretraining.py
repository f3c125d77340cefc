"""Token corpora on disk for language-model pretraining (capabilities of ``src/forgeline/data/pretraining.py``).

A split is one flat ``<split>.bin`` of token ids (uint16, or uint32 when the vocabulary needs it -- the
``meta.pkl`` written by corpus preparation says which).  ``MemmapCorpus`` maps it read-only and serves
next-token windows ``x = t[s : s + T]``, ``y = t[s + 1 : s + T + 1]``:

* ``sample_batch`` draws ``B`` random starts and gathers all ``B x (T + 1)`` tokens with one fancy index
  of the memmap into a reusable pinned staging buffer, then issues one asynchronous host-to-device copy
  (``x`` and ``y`` are views of the same device window tensor);
* iteration walks the non-overlapping windows that start at multiples of ``T`` (one slice of the map each,
  converted to int64).
"""

from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, Iterator, Optional, Tuple

import numpy as np
import torch

from rl_project_b200.core.errors import DatasetError
from rl_project_b200.data.tokenizers import load_tokenizer_metadata

_WIDE = np.dtype(np.uint32)
_NARROW = np.dtype(np.uint16)


def detect_token_dtype(data_dir: str | Path) -> np.dtype:
    """The id width recorded for a prepared corpus: uint32 for tiktoken or vocabularies over 65535."""
    if not (Path(data_dir) / "meta.pkl").exists():
        return _NARROW
    meta = load_tokenizer_metadata(data_dir)
    wide = meta.get("tokenizer_type") == "tiktoken" or int(meta.get("vocab_size", 0)) > np.iinfo(np.uint16).max
    return _WIDE if wide else _NARROW


class MemmapCorpus:
    kind = "pretraining"

    def __init__(self, data_dir: str | Path, split: str, block_size: int, dtype: Optional[np.dtype] = None):
        self.data_dir, self.split, self.block_size = Path(data_dir), split, block_size
        path = self.data_dir / f"{split}.bin"
        if not path.exists():
            raise DatasetError(f"Token file not found: {path}", hint="Prepare the corpus (`data prepare`) first.")
        self.dtype = np.dtype(dtype) if dtype is not None else detect_token_dtype(self.data_dir)
        self.data = np.memmap(path, dtype=self.dtype, mode="r")
        if self.data.shape[0] <= block_size + 1:
            raise DatasetError(f"{path} has {self.data.shape[0]} tokens; need more than "
                               f"block_size+1={block_size + 1}")
        self._offsets = np.arange(block_size + 1, dtype=np.int64)
        self._staging: Dict[int, Tuple[torch.Tensor, Any]] = {}  # batch size -> (pinned [B, T + 1], copy event)

    def __len__(self) -> int:
        return self.data.shape[0] - self.block_size - 1

    @property
    def n_tokens(self) -> int:
        return int(self.data.shape[0])

    def _windows(self, starts: np.ndarray) -> np.ndarray:
        return np.asarray(self.data[starts[:, None] + self._offsets[None, :]], dtype=np.int64)

    def sample_batch(self, batch_size: int, device: torch.device | str = "cpu",
                     generator: Optional[torch.Generator] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        starts = torch.randint(self.data.shape[0] - self.block_size, (batch_size,), generator=generator).numpy()
        win = self._windows(starts)
        dev = torch.device(device)
        if dev.type != "cuda":
            t = torch.from_numpy(win)
            return t[:, :-1], t[:, 1:]
        buf, done = self._staging.get(batch_size, (None, None))
        if buf is None:
            buf = torch.empty(win.shape, dtype=torch.long, pin_memory=True)
        elif done is not None:
            done.synchronize()  # the previous copy out of this buffer has finished reading it
        buf.numpy()[...] = win
        t = buf.to(dev, non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(dev))
        self._staging[batch_size] = (buf, done)
        return t[:, :-1], t[:, 1:]

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        T = self.block_size
        n = -(-len(self) // T)  # windows starting at 0, T, 2T, ... below len(self)
        for k in range(n):
            w = torch.from_numpy(np.asarray(self.data[k * T:(k + 1) * T + 1], dtype=np.int64))
            yield w[:-1], w[1:]


def write_token_file(tokens: np.ndarray, path: str | Path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tokens.tofile(path)
    return path
