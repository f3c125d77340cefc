"""Optimizer construction (``src/forgeline/training/common/optim.py:11-30``):
decay only on matrices (``dim >= 2``) by default.  CUDA parameters get the
fused multi-tensor sm_100a AdamW with fp32 master weights; CPU parameters get
torch's AdamW/Adam with identical hyper-parameters."""

from __future__ import annotations

from typing import Iterable, List

import torch

from rl_project_b200.core.config import OptimizerConfig


def param_groups(params: List[torch.nn.Parameter], cfg: OptimizerConfig) -> List[dict]:
    if not cfg.decay_only_matrices:
        return [{"params": params, "weight_decay": cfg.weight_decay}]
    decay = [p for p in params if p.dim() >= 2]
    rest = [p for p in params if p.dim() < 2]
    groups = [{"params": decay, "weight_decay": cfg.weight_decay}]
    if rest:
        groups.append({"params": rest, "weight_decay": 0.0})
    return groups


def build_optimizer(params: Iterable[torch.nn.Parameter], cfg: OptimizerConfig,
                    device: torch.device) -> torch.optim.Optimizer:
    params = [p for p in params if p.requires_grad]
    if not params:
        raise ValueError("no trainable parameters")
    groups = param_groups(params, cfg)
    betas = (cfg.beta1, cfg.beta2)
    on_gpu = params[0].is_cuda
    if on_gpu and cfg.fused != "never":
        from rl_project_b200.ops.optim import FusedAdamW

        return FusedAdamW(groups, lr=cfg.learning_rate, betas=betas, eps=cfg.eps, decoupled=(cfg.name == "adamw"))
    cls = torch.optim.Adam if cfg.name == "adam" else torch.optim.AdamW
    return cls(groups, lr=cfg.learning_rate, betas=betas, eps=cfg.eps)
