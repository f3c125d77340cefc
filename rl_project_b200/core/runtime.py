"""Where a run executes and how it is seeded (the behaviour of ``src/forgeline/core/runtime.py:22-100``).

* ``resolve_device``: under a launcher with CUDA the process's ``LOCAL_RANK`` GPU; ``auto`` prefers CUDA, then
  Apple MPS, then CPU; an explicit ``cuda`` without CUDA is a configuration error.
* ``resolve_dtype``: ``auto`` is bf16 on CUDA (fp16 on GPUs without bf16) and fp32 elsewhere.
* ``seed_everything`` / ``rng_state`` / ``set_rng_state``: every generator a run draws from -- Python's, NumPy's,
  torch's host generator and every CUDA device's -- captured and restored as one dict (checkpoints store it).
"""

from __future__ import annotations

import os
import random
from contextlib import nullcontext
from typing import Any, Callable, ContextManager, Dict, Tuple

import numpy as np
import torch

from rl_project_b200.core.errors import ConfigError

DTYPE_MAP = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _auto_device() -> torch.device:
    if torch.cuda.is_available():
        return torch.device("cuda")
    mps = getattr(torch.backends, "mps", None)
    return torch.device("mps") if mps is not None and mps.is_available() else torch.device("cpu")


def resolve_device(requested: str = "auto", *, distributed: bool = False) -> torch.device:
    if distributed and torch.cuda.is_available():
        return torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    dev = _auto_device() if requested == "auto" else torch.device(requested)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise ConfigError("device=cuda requested but CUDA is not available", hint="Use device=cpu or auto.")
    return dev


def resolve_dtype(requested: str, device: torch.device) -> torch.dtype:
    if requested == "auto":
        if device.type != "cuda":
            return torch.float32
        return torch.bfloat16 if torch.cuda.is_bf16_supported() else torch.float16
    try:
        return DTYPE_MAP[requested]
    except KeyError:
        raise ConfigError(f"Unknown dtype {requested!r}; expected one of {sorted(DTYPE_MAP)}") from None


def autocast_context(device: torch.device, dtype: torch.dtype) -> ContextManager[Any]:
    """Autocast for reduced-precision compute where it applies (CUDA fp16 / bf16, CPU bf16), else a no-op."""
    half = dtype in (torch.bfloat16, torch.float16)
    if (device.type == "cuda" and half) or (device.type == "cpu" and dtype == torch.bfloat16):
        return torch.amp.autocast(device_type=device.type, dtype=dtype)
    return nullcontext()


# name -> (capture, restore) of one generator family; CUDA only when present
_GENERATORS: Dict[str, Tuple[Callable[[], Any], Callable[[Any], None]]] = {
    "python": (random.getstate, random.setstate),
    "numpy": (np.random.get_state, np.random.set_state),
    "torch": (torch.get_rng_state, torch.set_rng_state),
    "cuda": (torch.cuda.get_rng_state_all, torch.cuda.set_rng_state_all),
}


def seed_everything(seed: int, *, deterministic: bool = False) -> None:
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)  # also every CUDA device
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)


def rng_state() -> Dict[str, Any]:
    return {name: capture() for name, (capture, _) in _GENERATORS.items()
            if name != "cuda" or torch.cuda.is_available()}


def set_rng_state(state: Dict[str, Any]) -> None:
    for name, (_, restore) in _GENERATORS.items():
        if name in state and (name != "cuda" or torch.cuda.is_available()):
            restore(state[name])


def has_cuda() -> bool:
    return torch.cuda.is_available()


def cuda_device_count() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0
