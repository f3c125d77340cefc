"""tcgen05/TMEM GEMM entry points (csrc/gemm_tcgen05.cu); disabled until the kernel is built."""

from __future__ import annotations

import torch


def enabled() -> bool:
    return False


def supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    return False


def gemm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:  # pragma: no cover
    raise NotImplementedError


def linear(x, w, bias=None):  # pragma: no cover
    raise NotImplementedError
