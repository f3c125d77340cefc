"""Tokenised (prompt, response) pairs for supervised fine-tuning.

Each record becomes ``(prompt ids, target ids)`` fitted into ``max_length`` tokens: the response is cut
to the room the prompt leaves; a prompt that fills the window keeps its first ``max_length - 1`` tokens
and one response token, so every example trains on at least one target (the reference's truncation
rule, ``src/forgeline/data/supervised.py``).  Examples are stored packed (``PackedExamples``).
"""

from __future__ import annotations

from collections.abc import Sequence as _SequenceABC
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

from rl_project_b200.data.packed import PackedExamples
from rl_project_b200.data.records import ReadReport, SFTRecord, read_jsonl


def fit_pair(prompt: List[int], target: List[int], max_length: int) -> Optional[Tuple[List[int], List[int]]]:
    """Cut ``(prompt, target)`` to ``max_length`` tokens as described above (None if under two tokens)."""
    if len(prompt) >= max_length:  # the prompt fills the window: keep one target token after it
        prompt, target = prompt[:max_length - 1], target[:1]
    else:
        target = target[:max_length - len(prompt)]
    return (prompt, target) if len(prompt) + len(target) >= 2 else None


class SupervisedDataset(_SequenceABC):
    kind = "supervised"

    def __init__(self, records: Sequence[SFTRecord], tokenizer, max_length: int = 512, response_suffix: str = ""):
        self.records = list(records)
        self.tokenizer = tokenizer
        self.max_length = max_length
        self.response_suffix = response_suffix
        pairs = (fit_pair(tokenizer.encode(r.prompt), tokenizer.encode(r.response + response_suffix), max_length)
                 for r in self.records)
        self._packed = PackedExamples(("prompt", "target"), (p for p in pairs if p is not None))

    @classmethod
    def from_jsonl(cls, path: str | Path, tokenizer, max_length: int = 512, on_error: str = "raise",
                   report: Optional[ReadReport] = None) -> "SupervisedDataset":
        return cls(read_jsonl(path, SFTRecord, on_error=on_error, report=report), tokenizer, max_length)

    def __len__(self) -> int:
        return len(self._packed)

    def __getitem__(self, i):
        return self._packed[i]
