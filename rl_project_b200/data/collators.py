"""Batch assembly from token lists (capabilities of ``src/forgeline/data/collators.py``).

Everything is built from one flat token tensor and a lengths vector: a ``[B, W]`` boolean occupancy mask
(``arange(W) < length``, flipped for left padding) places the flat tokens with a single masked assignment,
and the supervised targets come from comparing column indices against per-row bounds -- no per-row Python
slicing of tensors.  ``IGNORE_INDEX = -1`` is the native loss's ignore index.

Supervised layout: the row ``[prompt | response]`` (cut to ``max_length``) is shifted by one; target ``j``
is token ``j + 1``, kept only where ``prompt_length - 1 <= j < length - 1`` (``mask_prompt``) or
``j < length - 1`` (not masking the prompt).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from rl_project_b200.core.errors import DatasetError

IGNORE_INDEX = -1


def _occupancy(lengths: torch.Tensor, width: int, side: str) -> torch.Tensor:
    cols = torch.arange(width)
    if side == "right":
        return cols[None, :] < lengths[:, None]
    if side == "left":
        return cols[None, :] >= (width - lengths)[:, None]
    raise DatasetError("padding side must be 'left' or 'right'")


def _flat(seqs: Sequence[Sequence[int]]) -> Tuple[torch.Tensor, torch.Tensor]:
    lengths = torch.tensor([len(s) for s in seqs], dtype=torch.long)
    flat = torch.tensor([t for s in seqs for t in s], dtype=torch.long)
    return flat, lengths


def pad_sequences(seqs: Sequence[Sequence[int]], pad_value: int, side: str = "right") -> Tuple[torch.Tensor, torch.Tensor]:
    """``(ids [B, W], attention_mask [B, W])`` with ``W`` the longest sequence; empty rows are all padding."""
    flat, lengths = _flat(seqs)
    width = int(lengths.max()) if len(seqs) else 0
    occ = _occupancy(lengths, width, side)
    ids = torch.full((len(seqs), width), pad_value, dtype=torch.long)
    ids[occ] = flat  # row-major order of the mask matches the concatenation order
    return ids, occ.long()


@dataclass
class SupervisedBatch:
    input_ids: torch.Tensor
    targets: torch.Tensor
    attention_mask: torch.Tensor
    prompt_lengths: List[int]

    def to(self, device, non_blocking: bool = False) -> "SupervisedBatch":
        mv = lambda t: t.to(device, non_blocking=non_blocking)  # noqa: E731
        return SupervisedBatch(mv(self.input_ids), mv(self.targets), mv(self.attention_mask), self.prompt_lengths)

    def micro(self, i: int, n: int) -> "SupervisedBatch":
        """Every ``n``-th row from row ``i`` (strided, so micro-batches mix short and long rows alike)."""
        sl = slice(i, None, n)
        return SupervisedBatch(self.input_ids[sl], self.targets[sl], self.attention_mask[sl], self.prompt_lengths[sl])


def collate_supervised(examples: Sequence[Tuple[List[int], List[int]]], pad_value: int = 0,
                       max_length: int | None = None, mask_prompt: bool = True) -> SupervisedBatch:
    rows = [(list(p) + list(r))[:max_length] if max_length is not None else list(p) + list(r) for p, r in examples]
    if any(len(x) < 2 for x in rows):
        raise DatasetError("supervised example must contain at least two tokens")
    plens = [min(len(p), len(x)) for (p, _), x in zip(examples, rows)]
    ids, mask = pad_sequences(rows, pad_value, "right")
    lengths = mask.sum(1)
    cols = torch.arange(ids.shape[1] - 1)[None, :]
    lo = (torch.tensor(plens, dtype=torch.long) - 1).clamp_min(0) if mask_prompt else torch.zeros_like(lengths)
    keep = (cols >= lo[:, None]) & (cols < (lengths - 1)[:, None])
    targets = torch.where(keep, ids[:, 1:], torch.full_like(ids[:, 1:], IGNORE_INDEX))
    return SupervisedBatch(ids[:, :-1], targets, mask[:, :-1], plens)


def collate_lm(examples: Sequence[Tuple[torch.Tensor, torch.Tensor]]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Stack equal-length ``(x, y)`` windows."""
    xs, ys = zip(*examples)
    return torch.stack(xs), torch.stack(ys)


def collate_preference(examples: Sequence[Dict[str, List[int]]], pad_value: int = 0) -> Dict[str, torch.Tensor]:
    """Prompts left-padded (their last token adjacent to the continuation); chosen / rejected right-padded."""
    out: Dict[str, torch.Tensor] = {}
    for key, side in (("prompt", "left"), ("chosen", "right"), ("rejected", "right")):
        ids, mask = pad_sequences([e[key] for e in examples], pad_value, side)
        out[key] = ids
        if key != "prompt":
            out[f"{key}_mask"] = mask
    return out
