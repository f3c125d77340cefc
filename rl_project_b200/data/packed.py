"""Compact storage for tokenised datasets: each field's sequences of every example live in one flat
int32 array with an offsets array, instead of one Python list per example (a million-example SFT set
costs tens of MB here against gigabytes of list objects).  ``PackedExamples[i]`` returns the example's
fields as lists of ints, which is what the collators consume."""

from __future__ import annotations

from collections.abc import Sequence as _SequenceABC
from typing import Dict, Iterable, List, Sequence, Tuple

import numpy as np


class PackedExamples(_SequenceABC):
    """Examples with a fixed set of named token fields, packed field by field."""

    def __init__(self, fields: Sequence[str], rows: Iterable[Sequence[Sequence[int]]]):
        self.fields = tuple(fields)
        flat: List[List[int]] = [[] for _ in self.fields]
        lens: List[List[int]] = [[] for _ in self.fields]
        for row in rows:
            for f, seq in enumerate(row):
                flat[f].extend(seq)
                lens[f].append(len(seq))
        self._data = [np.asarray(x, dtype=np.int32) for x in flat]
        self._off = [np.concatenate(([0], np.cumsum(np.asarray(n, dtype=np.int64)))) for n in lens]

    def __len__(self) -> int:
        return len(self._off[0]) - 1 if self._off else 0

    def field(self, f: int, i: int) -> List[int]:
        lo, hi = self._off[f][i], self._off[f][i + 1]
        return self._data[f][lo:hi].tolist()

    def __getitem__(self, i: int) -> Tuple[List[int], ...]:
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        n = len(self)
        if not -n <= i < n:
            raise IndexError(i)
        i %= n
        return tuple(self.field(f, i) for f in range(len(self.fields)))

    def as_dict(self, i: int) -> Dict[str, List[int]]:
        return dict(zip(self.fields, self[i]))

    def token_count(self) -> int:
        return int(sum(d.size for d in self._data))
