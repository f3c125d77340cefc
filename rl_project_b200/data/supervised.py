"""Tokenised (prompt, response) pairs for SFT (``src/forgeline/data/supervised.py``)."""

from __future__ import annotations

from pathlib import Path
from typing import Iterator, List, Optional, Sequence, Tuple

from rl_project_b200.data.records import ReadReport, SFTRecord, read_jsonl


class SupervisedDataset:
    kind = "supervised"

    def __init__(self, records: Sequence[SFTRecord], tokenizer, max_length: int = 512, response_suffix: str = ""):
        self.records = list(records)
        self.tokenizer = tokenizer
        self.max_length = max_length
        self.response_suffix = response_suffix
        self._examples: List[Tuple[List[int], List[int]]] = []
        for r in self.records:
            p = tokenizer.encode(r.prompt)
            t = tokenizer.encode(r.response + response_suffix)
            room = max_length - len(p)
            if room < 1:
                p, t = p[: max_length - 1], t[:1]
            else:
                t = t[:room]
            if len(p) + len(t) >= 2:
                self._examples.append((p, t))

    @classmethod
    def from_jsonl(cls, path: str | Path, tokenizer, max_length: int = 512, on_error: str = "raise",
                   report: Optional[ReadReport] = None) -> "SupervisedDataset":
        return cls(read_jsonl(path, SFTRecord, on_error=on_error, report=report), tokenizer, max_length)

    def __len__(self) -> int:
        return len(self._examples)

    def __getitem__(self, i: int):
        return self._examples[i]

    def __iter__(self) -> Iterator[Tuple[List[int], List[int]]]:
        return iter(self._examples)
