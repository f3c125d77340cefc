"""Learning-rate schedules (``src/forgeline/training/common/schedule.py``):
cosine with linear warm-up (default), warm-up-stable-decay, constant, linear decay."""

from __future__ import annotations

import math

from rl_project_b200.core.config import ScheduleConfig


def _warm(step: int, peak: float, warmup: int):
    return peak * step / warmup if warmup > 0 and step < warmup else None


def learning_rate_at(step: int, peak_lr: float, cfg: ScheduleConfig) -> float:
    w = _warm(step, peak_lr, cfg.warmup_steps)
    if w is not None:
        return w
    if cfg.name == "constant":
        return peak_lr
    if cfg.name == "wsd":
        stable_end = int(cfg.decay_steps * cfg.wsd_stable_fraction)
        if step < stable_end:
            return peak_lr
        frac = min((step - stable_end) / max(1, cfg.decay_steps - stable_end), 1.0)
        return cfg.min_lr + 0.5 * (1.0 + math.cos(math.pi * frac)) * (peak_lr - cfg.min_lr)
    if cfg.name == "linear_decay":
        if step >= cfg.decay_steps:
            return cfg.min_lr
        frac = (step - cfg.warmup_steps) / max(1, cfg.decay_steps - cfg.warmup_steps)
        return peak_lr + (cfg.min_lr - peak_lr) * min(max(frac, 0.0), 1.0)
    if step > cfg.decay_steps:
        return cfg.min_lr
    frac = (step - cfg.warmup_steps) / max(1, cfg.decay_steps - cfg.warmup_steps)
    return cfg.min_lr + 0.5 * (1.0 + math.cos(math.pi * frac)) * (peak_lr - cfg.min_lr)
