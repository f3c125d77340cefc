"""Dense GEMMs of the model.

``linear`` (every linear layer, with its backward) and ``matmul_nt`` /
``matmul_nn`` / ``matmul_tn`` (the LM head's products) run this library's
tcgen05 GEMM (csrc/gemm_2sm.cu) on sm_100a as ``RLB_GEMM`` selects: by default
(``hybrid``) the forward products run the own kernel and the gradient products
cuBLAS; ``tcgen05`` runs all of them on the own kernel, ``cublas`` none.
"""

from __future__ import annotations

import os

import torch

def _own(a: torch.Tensor, b: torch.Tensor) -> bool:
    if not (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.dim() == 2 and b.dim() == 2):
        return False
    from rl_project_b200.ops import gemm

    return gemm.enabled() and all(x % 8 == 0 for x in (*a.shape, *b.shape)) and \
        a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0


def matmul_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M, K] @ b [N, K]^T``."""
    if _own(a, b):
        from rl_project_b200.ops import gemm

        if gemm.supported(a, b):
            return gemm.gemm_nt(a, b)
    return a @ b.t()


def matmul_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M, K] @ b [K, N]`` (b read as stored; the LM head's input gradient)."""
    from rl_project_b200.ops import gemm

    if _own(a, b) and gemm.dgrad_own():
        from rl_project_b200.ops import gemm

        return gemm.gemm_nn(a, b)
    return a @ b


def matmul_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [K, M]^T @ b [K, N]`` (both read as stored; the LM head's weight gradient)."""
    from rl_project_b200.ops import gemm

    if _own(a, b) and gemm.wgrad_own():
        from rl_project_b200.ops import gemm

        return gemm.gemm_tn(a, b)
    return a.t() @ b


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w^T (+ bias)`` for ``x [..., K]``, ``w [N, K]``."""
    if x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16:
        from rl_project_b200.ops import gemm

        if gemm.enabled():
            return gemm.linear(x, w, bias)
    return torch.nn.functional.linear(x, w, bias)
