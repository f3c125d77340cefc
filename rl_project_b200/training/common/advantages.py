"""Advantage estimators (``src/forgeline/training/common/advantages.py``)."""

from __future__ import annotations

from typing import Tuple

import torch


def compute_gae(rewards: torch.Tensor, values: torch.Tensor, gamma: float = 0.99,
                lam: float = 0.95) -> Tuple[torch.Tensor, torch.Tensor]:
    T = rewards.shape[0]
    adv = torch.zeros(T, dtype=torch.float32)
    run = 0.0
    for t in range(T - 1, -1, -1):
        delta = float(rewards[t]) + gamma * float(values[t + 1]) - float(values[t])
        run = delta + gamma * lam * run
        adv[t] = run
    return adv, adv + values[:T].float()


def normalize_advantages(adv: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    if adv.numel() <= 1:
        return torch.zeros_like(adv)
    return (adv - adv.mean()) / (adv.std() + eps)


def group_relative_advantages(rewards: torch.Tensor, eps: float = 1e-8, clamp_std: bool = False) -> torch.Tensor:
    if rewards.numel() <= 1:
        return torch.zeros_like(rewards)
    sd = rewards.std()
    sd = sd.clamp(min=eps) if clamp_std else sd + eps
    return (rewards - rewards.mean()) / sd


def grouped_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-8,
                       clamp_std: bool = False) -> torch.Tensor:
    """Vectorised ``group_relative_advantages`` over consecutive groups of ``group_size``."""
    r = rewards.view(-1, group_size).float()
    if group_size <= 1:
        return torch.zeros_like(rewards, dtype=torch.float32)
    sd = r.std(dim=1, keepdim=True)
    sd = sd.clamp(min=eps) if clamp_std else sd + eps
    return ((r - r.mean(dim=1, keepdim=True)) / sd).view(-1)
