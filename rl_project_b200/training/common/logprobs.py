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

from typing import List, Optional, Sequence, Tuple

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


# ---------------------------------------------------------------- packed scoring of prompt + response rows
def pack_prompt_response(pairs: Sequence[Tuple[List[int], List[int]]], pad: int):
    """Right-padded ``inputs [N, T]`` and ``targets [N, T]`` (-1 outside each response): row ``i`` holds
    ``prompt + response`` shifted by one, so target ``t`` is the token that follows input ``t``.  Under causal
    attention the padding after a row cannot change its log-probs, so rows of different prompt lengths share
    one forward."""
    rows = [list(p) + list(r) for p, r in pairs]
    starts = torch.tensor([len(p) - 1 for p, _ in pairs])  # first input position that predicts a response token
    lengths = torch.tensor([len(x) - 1 for x in rows])
    T = int(lengths.max())
    flat = torch.full((len(rows), T + 1), pad, dtype=torch.long)
    for i, x in enumerate(rows):
        flat[i, :len(x)] = torch.as_tensor(x)
    cols = torch.arange(T)[None, :]
    inputs = torch.where(cols < lengths[:, None], flat[:, :-1], torch.full_like(flat[:, :-1], pad))
    in_response = (cols >= starts[:, None]) & (cols < lengths[:, None])
    targets = torch.where(in_response, flat[:, 1:], torch.full_like(flat[:, 1:], -1))
    return inputs, targets


def packed_response_logprobs(policy, trajectories, width: int, with_entropy: bool = False):
    """Response-aligned ``[N, width]`` log-probs (and entropies) of ``policy.model`` for every trajectory,
    from ONE packed forward through the fused LM-head kernel; positions past a response are unspecified
    (callers mask them)."""
    pairs = [(t.prompt_ids.tolist(), t.response_ids.tolist()) for t in trajectories]
    inputs, targets = pack_prompt_response(pairs, policy.pad_token_id)
    dev = policy.device
    inputs, targets = inputs.to(dev), targets.to(dev)
    ent = None
    if not with_entropy:
        lp = policy.token_logprobs(inputs, targets)
    elif hasattr(policy.model, "token_logprobs"):  # the native model: entropy from the same fused pass
        lp, ent = policy.model.token_logprobs(inputs, targets, with_entropy=True)
    else:  # other backends: from full logits
        logits = policy.token_logits(inputs).float()
        logp = logits.log_softmax(-1)
        lp = logp.gather(-1, targets.clamp(min=0)[..., None])[..., 0] * (targets >= 0)
        ent = -(logp.exp() * logp).sum(-1)
    starts = torch.tensor([len(p) - 1 for p, _ in pairs], device=dev)
    cols = (starts[:, None] + torch.arange(width, device=dev)[None, :]).clamp(max=lp.shape[1] - 1)
    return lp.float().gather(1, cols), (ent.float().gather(1, cols) if ent is not None else None)
