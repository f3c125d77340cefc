"""Advantage estimators (the estimators of ``src/forgeline/training/common/advantages.py``).

* ``compute_gae``: generalised advantage estimation, ``A_t = sum_k (gamma lambda)^k delta_{t+k}`` with
  ``delta_t = r_t + gamma V_{t+1} - V_t``, evaluated as one backward recurrence over a float64 array
  (``values`` has one more entry than ``rewards``: the bootstrap value); returns ``(A, A + V)``.
* group-relative advantages (GRPO): ``(r - mean) / (std + eps)`` within a group, or with the standard
  deviation floored at ``eps`` (``clamp_std``); ``grouped_advantages`` does every group of a flat reward
  vector at once.
"""

from __future__ import annotations

from typing import Tuple

import numpy as np
import torch


def compute_gae(rewards: torch.Tensor, values: torch.Tensor, gamma: float = 0.99,
                lam: float = 0.95) -> Tuple[torch.Tensor, torch.Tensor]:
    r = rewards.detach().double().cpu().numpy()
    v = values.detach().double().cpu().numpy()
    delta = r + gamma * v[1:len(r) + 1] - v[:len(r)]
    adv = np.empty_like(delta)
    acc, decay = 0.0, gamma * lam
    for t in range(len(delta) - 1, -1, -1):
        acc = delta[t] + decay * acc
        adv[t] = acc
    a = torch.from_numpy(adv).float()
    return a, a + values[:len(r)].float().cpu()


def _standardise(x: torch.Tensor, dim, eps: float, clamp_std: bool) -> torch.Tensor:
    sd = x.std(dim=dim, keepdim=dim is not None)
    sd = sd.clamp(min=eps) if clamp_std else sd + eps
    return (x - x.mean(dim=dim, keepdim=dim is not None)) / sd


def normalize_advantages(adv: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    return torch.zeros_like(adv) if adv.numel() <= 1 else _standardise(adv, None, eps, False)


def group_relative_advantages(rewards: torch.Tensor, eps: float = 1e-8, clamp_std: bool = False) -> torch.Tensor:
    return torch.zeros_like(rewards) if rewards.numel() <= 1 else _standardise(rewards, None, eps, clamp_std)


def grouped_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-8,
                       clamp_std: bool = False) -> torch.Tensor:
    """``group_relative_advantages`` of every consecutive group of ``group_size`` rewards at once."""
    if group_size <= 1:
        return torch.zeros_like(rewards, dtype=torch.float32)
    return _standardise(rewards.view(-1, group_size).float(), 1, eps, clamp_std).view(-1)
