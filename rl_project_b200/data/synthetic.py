"""Seeded synthetic data for every benchmark configuration.

* ``SyntheticSFTSource``: token ids uniform over the vocabulary, the first
  ``prompt_fraction`` of every sequence masked out of the loss (dense SFT).
* ``SyntheticPretrainSource``: uniform ids, every position supervised.
* ``addition_tasks``: ``"a+b="`` prompts with decimal-sum targets (tiny SFT->GRPO).
* ``random_prompts``: variable-length uniform-id prompts (GRPO rollouts).

Streams are a pure function of ``(seed, rank)`` so data-parallel ranks draw
different batches and every run is reproducible.  Host batches live in
pinned memory and are copied to the device asynchronously by ``collect``.
"""

from __future__ import annotations

import random
from typing import Dict, List, Optional, Tuple

import torch

from rl_project_b200.data.collators import IGNORE_INDEX, SupervisedBatch


class SyntheticSFTSource:
    def __init__(self, vocab_size: int, seq_len: int, batch_size: int, prompt_fraction: float = 0.25,
                 seed: int = 0, rank: int = 0, pin: bool = True, pool: int = 2):
        self.vocab_size = vocab_size
        self.seq_len = seq_len
        self.batch_size = batch_size
        self.prompt_len = int(seq_len * prompt_fraction)
        self.gen = torch.Generator().manual_seed(seed * 1_000_003 + rank)
        pin = pin and torch.cuda.is_available()
        # a small pool of distinct host batches, generated once (uniform ids are cheap to regenerate but
        # generating 32k ids per step on the host would dominate a tiny benchmark)
        self._pool: List[SupervisedBatch] = [self._make(pin) for _ in range(max(1, pool))]
        self._i = 0

    def _make(self, pin: bool) -> SupervisedBatch:
        toks = torch.randint(0, self.vocab_size, (self.batch_size, self.seq_len + 1), generator=self.gen)
        x = toks[:, :-1].contiguous()
        y = toks[:, 1:].contiguous()
        y[:, : max(self.prompt_len - 1, 0)] = IGNORE_INDEX
        mask = torch.ones_like(x)
        if pin:
            x, y, mask = x.pin_memory(), y.pin_memory(), mask.pin_memory()
        return SupervisedBatch(x, y, mask, [self.prompt_len] * self.batch_size)

    def next_batch(self) -> SupervisedBatch:
        b = self._pool[self._i % len(self._pool)]
        self._i += 1
        return b

    def bytes_per_batch(self) -> int:
        b = self._pool[0]
        return b.input_ids.numel() * 8 + b.targets.numel() * 8


class SyntheticPretrainSource:
    def __init__(self, vocab_size: int, seq_len: int, batch_size: int, seed: int = 0, rank: int = 0):
        self.gen = torch.Generator().manual_seed(seed * 7919 + rank)
        self.vocab_size, self.seq_len, self.batch_size = vocab_size, seq_len, batch_size

    def __iter__(self):
        return self

    def __next__(self) -> Tuple[torch.Tensor, torch.Tensor]:
        t = torch.randint(0, self.vocab_size, (self.batch_size, self.seq_len + 1), generator=self.gen)
        return t[:, :-1].contiguous(), t[:, 1:].contiguous()


def addition_tasks(n: int, seed: int = 0, lo: int = 0, hi: int = 99) -> List[Dict[str, str]]:
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        a, b = rng.randint(lo, hi), rng.randint(lo, hi)
        out.append({"prompt": f"{a}+{b}=", "answer": str(a + b), "response": str(a + b)})
    return out


def random_prompts(n: int, vocab_size: int, min_len: int, max_len: int, seed: int = 0) -> List[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (n,), generator=g).tolist()
    return [torch.randint(0, vocab_size, (L,), generator=g) for L in lens]
