"""Padding and batch assembly (``src/forgeline/data/collators.py``): right padding
for supervised batches with next-token targets, prompt masking with
``IGNORE_INDEX = -1`` (the native loss's ignore index), left-padded prompts
for preference batches."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from rl_project_b200.core.errors import DatasetError

IGNORE_INDEX = -1


def pad_sequences(seqs: Sequence[Sequence[int]], pad_value: int, side: str = "right") -> Tuple[torch.Tensor, torch.Tensor]:
    if side not in ("left", "right"):
        raise DatasetError("padding side must be 'left' or 'right'")
    width = max((len(s) for s in seqs), default=0)
    ids = torch.full((len(seqs), width), pad_value, dtype=torch.long)
    mask = torch.zeros((len(seqs), width), dtype=torch.long)
    for i, s in enumerate(seqs):
        n = len(s)
        if not n:
            continue
        sl = slice(0, n) if side == "right" else slice(width - n, width)
        ids[i, sl] = torch.as_tensor(list(s), dtype=torch.long)
        mask[i, sl] = 1
    return ids, mask


@dataclass
class SupervisedBatch:
    input_ids: torch.Tensor
    targets: torch.Tensor
    attention_mask: torch.Tensor
    prompt_lengths: List[int]

    def to(self, device, non_blocking: bool = False) -> "SupervisedBatch":
        return SupervisedBatch(self.input_ids.to(device, non_blocking=non_blocking),
                               self.targets.to(device, non_blocking=non_blocking),
                               self.attention_mask.to(device, non_blocking=non_blocking), self.prompt_lengths)

    def micro(self, i: int, n: int) -> "SupervisedBatch":
        sl = slice(i, None, n)
        return SupervisedBatch(self.input_ids[sl], self.targets[sl], self.attention_mask[sl], self.prompt_lengths[sl])


def collate_supervised(examples: Sequence[Tuple[List[int], List[int]]], pad_value: int = 0,
                       max_length: int | None = None, mask_prompt: bool = True) -> SupervisedBatch:
    seqs, plens = [], []
    for prompt, response in examples:
        full = list(prompt) + list(response)
        if max_length is not None:
            full = full[:max_length]
        if len(full) < 2:
            raise DatasetError("supervised example must contain at least two tokens")
        seqs.append(full)
        plens.append(min(len(prompt), len(full)))
    ids, mask = pad_sequences(seqs, pad_value, "right")
    targets = ids[:, 1:].clone()
    targets[mask[:, 1:] == 0] = IGNORE_INDEX
    if mask_prompt:
        for i, p in enumerate(plens):
            targets[i, : max(p - 1, 0)] = IGNORE_INDEX
    return SupervisedBatch(ids[:, :-1], targets, mask[:, :-1], plens)


def collate_lm(examples: Sequence[Tuple[torch.Tensor, torch.Tensor]]) -> Tuple[torch.Tensor, torch.Tensor]:
    return torch.stack([x for x, _ in examples]), torch.stack([y for _, y in examples])


def collate_preference(examples: Sequence[Dict[str, List[int]]], pad_value: int = 0) -> Dict[str, torch.Tensor]:
    prompts, _ = pad_sequences([e["prompt"] for e in examples], pad_value, "left")
    chosen, cmask = pad_sequences([e["chosen"] for e in examples], pad_value, "right")
    rejected, rmask = pad_sequences([e["rejected"] for e in examples], pad_value, "right")
    return {"prompt": prompts, "chosen": chosen, "chosen_mask": cmask, "rejected": rejected, "rejected_mask": rmask}
