"""Masked reductions over token positions and the KL / entropy estimators of the RL objectives (the functions
of ``src/forgeline/training/common/logprobs.py``).

All reductions run over the last dimension by default; a ``mask`` of 0 / 1 (any dtype) selects the positions
that count and a masked mean divides by the number of selected positions (at least 1).  The sequence-level KL
estimators compare per-token log-probs of the reference (``ref_lp``) and the policy (``new_lp``):

* ``logprob_diff``: mean of ``ref - new`` over the sequence, then clamped below at ``clamp_min`` -- the clamp
  applies after the average, as in the reference (``None`` disables it);
* ``k3``: mean of ``exp(d) - d - 1`` with ``d = ref - new`` (non-negative per token).
"""

from __future__ import annotations

from typing import Optional

import torch


def _reduce(x: torch.Tensor, mask: Optional[torch.Tensor], dim: int, mean: bool) -> torch.Tensor:
    if mask is None:
        return x.mean(dim=dim) if mean else x.sum(dim=dim)
    m = mask.to(x.dtype)
    total = (x * m).sum(dim=dim)
    return total / m.sum(dim=dim).clamp(min=1.0) if mean else total


def masked_mean(x: torch.Tensor, mask: Optional[torch.Tensor], dim: int = -1) -> torch.Tensor:
    return _reduce(x, mask, dim, True)


def masked_sum(x: torch.Tensor, mask: Optional[torch.Tensor], dim: int = -1) -> torch.Tensor:
    return _reduce(x, mask, dim, False)


def reduce_logprobs(token_lp: torch.Tensor, mask: Optional[torch.Tensor], reduction: str) -> torch.Tensor:
    if reduction not in ("sum", "mean"):
        raise ValueError(f"reduction must be sum|mean, got {reduction!r}")
    return _reduce(token_lp, mask, -1, reduction == "mean")


def kl_logprob_diff(ref_lp: torch.Tensor, new_lp: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    clamp_min: Optional[float] = 0.0) -> torch.Tensor:
    kl = masked_mean(ref_lp - new_lp, mask)
    return kl if clamp_min is None else kl.clamp(min=clamp_min)


def kl_k3(ref_lp: torch.Tensor, new_lp: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    d = ref_lp - new_lp
    return masked_mean(torch.exp(d) - d - 1.0, mask)


def kl_full_distribution(new_logits: torch.Tensor, ref_logits: torch.Tensor) -> torch.Tensor:
    """``KL(new || ref)`` per position from full logits (fp32)."""
    new_lp = torch.log_softmax(new_logits.float(), -1)
    ref_lp = torch.log_softmax(ref_logits.float(), -1)
    return torch.sum(new_lp.exp() * (new_lp - ref_lp), dim=-1)


def entropy_from_logits(logits: torch.Tensor) -> torch.Tensor:
    lp = torch.log_softmax(logits.float(), -1)
    return -torch.sum(lp.exp() * lp, dim=-1)
