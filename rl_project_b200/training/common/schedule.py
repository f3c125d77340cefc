"""Learning-rate schedules (the schedules of ``src/forgeline/training/common/schedule.py``).

Every schedule is a linear warm-up to the peak over ``warmup_steps`` followed by a shape evaluated on the
decay phase.  A shape maps the fraction ``f`` of its decay window already elapsed to a factor ``s`` in
``[0, 1]``, and the rate is ``min_lr + s * (peak - min_lr)`` (``constant`` ignores ``min_lr``):

* ``cosine`` (default): window ``[warmup_steps, decay_steps]``, ``s = (1 + cos(pi f)) / 2``, ``min_lr`` after;
* ``linear_decay``: same window, ``s = 1 - f``;
* ``wsd`` (warm-up, stable, decay): the rate holds the peak until ``wsd_stable_fraction * decay_steps``, then
  the cosine shape over the rest of ``decay_steps``;
* ``constant``: the peak.
"""

from __future__ import annotations

import math
from typing import Callable, Dict, Tuple

from rl_project_b200.core.config import ScheduleConfig


def _cosine(f: float) -> float:
    return 0.5 * (1.0 + math.cos(math.pi * f))


def _window(step: int, start: int, end: int) -> float:
    """Elapsed fraction of ``[start, end]`` at ``step``, clamped to [0, 1]."""
    return min(max((step - start) / max(1, end - start), 0.0), 1.0)


# name -> (window start as a function of the config, decay shape)
_SHAPES: Dict[str, Tuple[Callable[[ScheduleConfig], int], Callable[[float], float]]] = {
    "cosine": (lambda c: c.warmup_steps, _cosine),
    "linear_decay": (lambda c: c.warmup_steps, lambda f: 1.0 - f),
    "wsd": (lambda c: int(c.decay_steps * c.wsd_stable_fraction), _cosine),
}


def learning_rate_at(step: int, peak_lr: float, cfg: ScheduleConfig) -> float:
    if cfg.warmup_steps > 0 and step < cfg.warmup_steps:
        return peak_lr * step / cfg.warmup_steps
    if cfg.name == "constant":
        return peak_lr
    start_of, shape = _SHAPES.get(cfg.name, _SHAPES["cosine"])
    start = start_of(cfg)
    if step < start:  # wsd's stable phase
        return peak_lr
    if step > cfg.decay_steps:
        return cfg.min_lr
    return cfg.min_lr + shape(_window(step, start, cfg.decay_steps)) * (peak_lr - cfg.min_lr)
