"""Masked reductions and KL / entropy estimators (``src/forgeline/training/common/logprobs.py``)."""

from __future__ import annotations

from typing import Optional

import torch


def masked_mean(x: torch.Tensor, mask: Optional[torch.Tensor], dim: int = -1) -> torch.Tensor:
    if mask is None:
        return x.mean(dim=dim)
    m = mask.to(x.dtype)
    return (x * m).sum(dim=dim) / m.sum(dim=dim).clamp(min=1.0)


def masked_sum(x: torch.Tensor, mask: Optional[torch.Tensor], dim: int = -1) -> torch.Tensor:
    return x.sum(dim=dim) if mask is None else (x * mask.to(x.dtype)).sum(dim=dim)


def reduce_logprobs(token_lp: torch.Tensor, mask: Optional[torch.Tensor], reduction: str) -> torch.Tensor:
    if reduction == "sum":
        return masked_sum(token_lp, mask)
    if reduction == "mean":
        return masked_mean(token_lp, mask)
    raise ValueError(f"reduction must be sum|mean, got {reduction!r}")


def kl_logprob_diff(ref_lp: torch.Tensor, new_lp: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    clamp_min: Optional[float] = 0.0) -> torch.Tensor:
    kl = masked_mean(ref_lp - new_lp, mask)
    return kl if clamp_min is None else kl.clamp(min=clamp_min)


def kl_k3(ref_lp: torch.Tensor, new_lp: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    d = ref_lp - new_lp
    return masked_mean(torch.exp(d) - d - 1.0, mask)


def kl_full_distribution(new_logits: torch.Tensor, ref_logits: torch.Tensor) -> torch.Tensor:
    a = torch.log_softmax(new_logits.float(), -1)
    b = torch.log_softmax(ref_logits.float(), -1)
    return (a.exp() * (a - b)).sum(-1)


def entropy_from_logits(logits: torch.Tensor) -> torch.Tensor:
    lp = torch.log_softmax(logits.float(), -1)
    return -(lp.exp() * lp).sum(-1)
