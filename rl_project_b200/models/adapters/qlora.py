"""QLoRA: frozen NF4 base weight + trainable LoRA (``src/forgeline/models/adapters/qlora.py``)."""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ModelError
from rl_project_b200.models.adapters.lora import DEFAULT_TARGET_MODULES, _children
from rl_project_b200.models.quantization.nf4 import NF4Linear


class QLoRALinear(nn.Module):
    def __init__(self, original: nn.Linear, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0):
        super().__init__()
        self.rank = rank
        self.alpha = alpha
        self.scaling = alpha / rank
        self.base = NF4Linear(original)
        dev = original.weight.device
        self.lora_A = nn.Parameter(torch.empty(original.in_features, rank, device=dev))
        self.lora_B = nn.Parameter(torch.zeros(rank, original.out_features, device=dev))
        nn.init.kaiming_uniform_(self.lora_A, a=5 ** 0.5)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.enabled = True

    @property
    def in_features(self) -> int:
        return self.base.in_features

    @property
    def out_features(self) -> int:
        return self.base.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.base(x)
        if not self.enabled:
            return y
        return y + (self.dropout(x) @ self.lora_A.to(x.dtype) @ self.lora_B.to(x.dtype)) * self.scaling


def apply_qlora(model: nn.Module, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0,
                target_modules: Optional[Sequence[str]] = None) -> nn.Module:
    targets = list(target_modules) if target_modules else list(DEFAULT_TARGET_MODULES)
    for p in model.parameters():
        p.requires_grad = False
    hit = 0
    for _, parent, attr, child in _children(model):
        if isinstance(child, nn.Linear) and any(t in attr for t in targets):
            setattr(parent, attr, QLoRALinear(child, rank, alpha, dropout))
            hit += 1
    if not hit:
        raise ModelError(f"No linear layers matched target_modules={targets}")
    return model
