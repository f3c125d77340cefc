"""Index sampling for the algorithms' ``collect`` steps.

``EpochSampler`` draws dataset indices without replacement: a seeded shuffle of the whole dataset per
epoch, consumed in order across steps, so every example is seen once per epoch and a batch never repeats
an example unless the dataset is smaller than the batch.  Its state (generator, permutation, cursor) is
checkpointed through the trainer's data-state capture (attribute ``sampler``), so a resumed run draws the
same batches.
"""

from __future__ import annotations

import random
from typing import List


class EpochSampler:
    def __init__(self, n: int, seed: int = 0):
        if n <= 0:
            raise ValueError("cannot sample from an empty dataset")
        self.n = n
        self.rng = random.Random(seed)
        self._order: List[int] = []
        self._pos = 0
        self.epoch = 0

    def _refill(self) -> None:
        self._order = list(range(self.n))
        self.rng.shuffle(self._order)
        self._pos = 0
        self.epoch += 1

    def take(self, k: int) -> List[int]:
        """The next ``k`` indices (crossing into a new epoch as needed)."""
        out: List[int] = []
        while len(out) < k:
            if self._pos >= len(self._order):
                self._refill()
            m = min(k - len(out), len(self._order) - self._pos)
            out += self._order[self._pos:self._pos + m]
            self._pos += m
        return out
