"""RMSNorm module (``src/forgeline/models/transformer/norm.py:9-17``); kernel in csrc/norm.cu."""

from __future__ import annotations

import torch
import torch.nn as nn

from rl_project_b200.ops.norm import rms_norm


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)
