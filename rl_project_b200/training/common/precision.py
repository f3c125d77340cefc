"""Mixed precision policy.

bf16 on CUDA: parameters live in bf16 and the optimizer keeps fp32 masters
(no autocast, no per-op casts).  fp16 on CUDA: fp32 parameters under autocast
with a GradScaler (reference behaviour, ``src/forgeline/training/common/precision.py``).
fp32 / CPU: plain.
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Any, ContextManager

import torch

from rl_project_b200.core.config import PrecisionConfig
from rl_project_b200.core.runtime import autocast_context


class Precision:
    def __init__(self, cfg: PrecisionConfig, device: torch.device, dtype: torch.dtype):
        self.device = device
        self.dtype = dtype
        self.master_weights = device.type == "cuda" and dtype == torch.bfloat16
        want_scaler = cfg.grad_scaler == "on" or (cfg.grad_scaler == "auto" and device.type == "cuda"
                                                  and dtype == torch.float16)
        self.scaler = torch.amp.GradScaler("cuda", enabled=bool(want_scaler and device.type == "cuda"))

    def autocast(self) -> ContextManager[Any]:
        if self.master_weights:
            return nullcontext()
        return autocast_context(self.device, self.dtype)

    def backward(self, loss: torch.Tensor) -> None:
        self.scaler.scale(loss).backward()

    def unscale(self, optimizer: torch.optim.Optimizer) -> None:
        if self.scaler.is_enabled():
            self.scaler.unscale_(optimizer)

    def step(self, optimizer: torch.optim.Optimizer) -> None:
        self.scaler.step(optimizer)
        self.scaler.update()

    def state_dict(self) -> dict:
        return self.scaler.state_dict()

    def load_state_dict(self, state: dict) -> None:
        if state:
            self.scaler.load_state_dict(state)
