"""Tokenised preference pairs for DPO-style training.

The prompt keeps its last ``max_prompt_length`` tokens (the end of a prompt is what the responses follow);
each response keeps its first ``max_response_length``.  Pairs with an empty side are dropped.  Items are
``{"prompt", "chosen", "rejected"}`` id lists (reference: ``src/forgeline/data/preference.py``), stored
packed.
"""

from __future__ import annotations

from collections.abc import Sequence as _SequenceABC
from pathlib import Path
from typing import Dict, List, Optional, Sequence

from rl_project_b200.data.packed import PackedExamples
from rl_project_b200.data.records import PreferenceRecord, ReadReport, read_jsonl

_FIELDS = ("prompt", "chosen", "rejected")


class PreferenceDataset(_SequenceABC):
    kind = "preference"

    def __init__(self, records: Sequence[PreferenceRecord], tokenizer, max_prompt_length: int = 384,
                 max_response_length: int = 128):
        self.records = list(records)
        self.tokenizer = tokenizer
        enc = tokenizer.encode

        def triple(r: PreferenceRecord):
            return (enc(r.prompt)[-max_prompt_length:], enc(r.chosen)[:max_response_length],
                    enc(r.rejected)[:max_response_length])

        self._packed = PackedExamples(_FIELDS, (t for t in map(triple, self.records) if all(t)))

    @classmethod
    def from_jsonl(cls, path: str | Path, tokenizer, max_prompt_length: int = 384, max_response_length: int = 128,
                   on_error: str = "raise", report: Optional[ReadReport] = None) -> "PreferenceDataset":
        return cls(read_jsonl(path, PreferenceRecord, on_error=on_error, report=report), tokenizer,
                   max_prompt_length, max_response_length)

    def __len__(self) -> int:
        return len(self._packed)

    def __getitem__(self, i) -> Dict[str, List[int]]:
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        return self._packed.as_dict(i)
