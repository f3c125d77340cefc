"""Dense GEMMs of the model.

``matmul_nt(a, b) = a @ b^T`` is the one entry every linear layer goes
through.  On sm_100a it runs the tcgen05 GEMM in csrc/gemm_tcgen05.cu when
that kernel is enabled for the shape, otherwise cuBLAS (a plain library GEMM
with no fused epilogue).
"""

from __future__ import annotations

import os

import torch

_USE_TCGEN05 = os.environ.get("RLB_GEMM", "auto")


def matmul_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if a.is_cuda and _USE_TCGEN05 != "cublas":
        from rl_project_b200.ops import gemm

        if gemm.supported(a, b):
            return gemm.gemm_nt(a, b)
    return a @ b.t()


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w^T (+ bias)`` for ``x [..., K]``, ``w [N, K]``."""
    if x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16:
        from rl_project_b200.ops import gemm

        if gemm.enabled():
            return gemm.linear(x, w, bias)
    return torch.nn.functional.linear(x, w, bias)
