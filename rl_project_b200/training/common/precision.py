"""Numeric mode of a training run (the Trainer's backward / unscale / step hooks).

Three modes, chosen once from the compute dtype, the device and ``PrecisionConfig.grad_scaler``:

* ``master`` -- bf16 on CUDA: parameters and activations are bf16 and the optimizer keeps fp32 master
  weights, so nothing is autocast and nothing is scaled (bf16 has fp32's exponent range);
* ``scaled`` -- fp16 on CUDA (or ``grad_scaler="on"``): fp32 parameters under fp16 autocast with dynamic
  loss scaling (``torch.amp.GradScaler``), as ``src/forgeline/training/common/precision.py`` does;
* ``plain`` -- everything else (fp32, CPU): autocast only where the runtime asks for it, no scaling.

``state_dict`` is the scaler's state (empty unless scaled), stored in checkpoints as ``scaler_state``.
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Any, ContextManager, Dict

import torch

from rl_project_b200.core.config import PrecisionConfig
from rl_project_b200.core.runtime import autocast_context


def precision_mode(cfg: PrecisionConfig, device: torch.device, dtype: torch.dtype) -> str:
    cuda = device.type == "cuda"
    if cuda and dtype == torch.bfloat16:
        return "master"
    if cuda and (cfg.grad_scaler == "on" or (cfg.grad_scaler == "auto" and dtype == torch.float16)):
        return "scaled"
    return "plain"


class Precision:
    def __init__(self, cfg: PrecisionConfig, device: torch.device, dtype: torch.dtype):
        self.device, self.dtype = device, dtype
        self.mode = precision_mode(cfg, device, dtype)
        self.scaler = torch.amp.GradScaler("cuda") if self.mode == "scaled" else None

    @property
    def master_weights(self) -> bool:
        return self.mode == "master"

    def autocast(self) -> ContextManager[Any]:
        return nullcontext() if self.mode == "master" else autocast_context(self.device, self.dtype)

    def backward(self, loss: torch.Tensor) -> None:
        (self.scaler.scale(loss) if self.scaler is not None else loss).backward()

    def unscale(self, optimizer: torch.optim.Optimizer) -> None:
        """Bring gradients to their true scale before clipping (no-op unless scaled)."""
        if self.scaler is not None:
            self.scaler.unscale_(optimizer)

    def step(self, optimizer: torch.optim.Optimizer) -> None:
        if self.scaler is None:
            optimizer.step()
            return
        self.scaler.step(optimizer)  # skipped when the unscaled gradients hold inf / nan
        self.scaler.update()

    def state_dict(self) -> Dict[str, Any]:
        return self.scaler.state_dict() if self.scaler is not None else {}

    def load_state_dict(self, state: Dict[str, Any]) -> None:
        if state and self.scaler is not None:
            self.scaler.load_state_dict(state)
