"""QLoRA: a frozen NF4-quantised base weight plus a trainable low-rank adapter (the capability of
``src/forgeline/models/adapters/qlora.py``).  The adapter is the one of ``lora.py`` (fp32 ``lora_A`` /
``lora_B``, same state layout); the base is ``NF4Linear``, whose matmul dequantises inside the GEMM on B200."""

from __future__ import annotations

from typing import Optional, Sequence

import torch.nn as nn

from rl_project_b200.models.adapters.lora import LowRankAdapter, attach_adapters
from rl_project_b200.models.quantization.nf4 import NF4Linear


class QLoRALinear(LowRankAdapter):
    def __init__(self, original: nn.Linear, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0):
        super().__init__()
        self.base = NF4Linear(original)
        self._init_adapter(original.in_features, original.out_features, rank, alpha, dropout,
                           original.weight.device, None)

    @property
    def in_features(self) -> int:
        return self.base.in_features

    @property
    def out_features(self) -> int:
        return self.base.out_features

    def base_forward(self, x):
        return self.base(x)


def apply_qlora(model: nn.Module, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0,
                target_modules: Optional[Sequence[str]] = None) -> nn.Module:
    return attach_adapters(model, target_modules, lambda lin: QLoRALinear(lin, rank, alpha, dropout))
