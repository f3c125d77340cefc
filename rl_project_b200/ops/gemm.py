"""tcgen05/TMEM GEMM (csrc/gemm_tcgen05.cu) and the linear layer built on it.

One persistent warp-specialised kernel covers a linear layer's three GEMMs
without transposing anything:

* forward      ``y  = x  W^T``   A = x  [M, K] (K-major),   B = W [N, K] (K-major)
* input grad   ``dx = dy W``     A = dy [M, N] (K-major),   B = W stored [N, K] read MN-major
* weight grad  ``dW = dy^T x``   A = dy read MN-major,      B = x read MN-major

``RLB_GEMM`` selects the implementation of the model's plain linear layers:
``tcgen05`` (this kernel), ``cublas`` (torch.matmul) or ``auto`` (tcgen05
once the numerics self-check on the first call passed).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from rl_project_b200.ops._ext import available, native

_MODE = os.environ.get("RLB_GEMM", "cublas")
_checked: dict = {}


def _ok_ptr(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def gemm_nt(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``a [M, K] @ b[N, K]^T`` in bf16 (fp32 accumulate)."""
    M, K = a.shape
    N = b.shape[0]
    a = a.contiguous()
    b = b.contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    native().gemm(a, b, out, 0, 0, 0, M, N, K, K, K, out.stride(0), alpha, None)
    return out


def gemm_nn(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0) -> torch.Tensor:
    """``a [M, K] @ b [K, N]`` (b read MN-major, no transpose)."""
    M, K = a.shape
    N = b.shape[1]
    a = a.contiguous()
    b = b.contiguous()
    out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    native().gemm(a, b, out, 0, 1, 0, M, N, K, K, N, N, alpha, None)
    return out


def gemm_tn(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, out: Optional[torch.Tensor] = None,
            accumulate: bool = False) -> torch.Tensor:
    """``a [K, M]^T @ b [K, N]`` -> ``[M, N]`` (both read MN-major).  fp32 ``out`` + ``accumulate`` adds into it."""
    K, M = a.shape
    N = b.shape[1]
    a = a.contiguous()
    b = b.contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
        epi = 0
    else:
        epi = 2 if accumulate else (1 if out.dtype == torch.float32 else 0)
    native().gemm(a, b, out, 1, 1, epi, M, N, K, M, N, out.stride(0), alpha, None)
    return out


def _shape_ok(x2: torch.Tensor, w: torch.Tensor) -> bool:
    M, K = x2.shape
    N = w.shape[0]
    return K % 8 == 0 and N % 8 == 0 and M % 8 == 0 and M > 0 and _ok_ptr(x2) and _ok_ptr(w)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, w):
        ctx.save_for_backward(x2, w)
        return gemm_nt(x2, w)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm_nn(dy, w) if ctx.needs_input_grad[0] else None
        dw = gemm_tn(dy, x2) if ctx.needs_input_grad[1] else None
        return dx, dw


def _self_check(device: torch.device) -> bool:
    key = (device.type, device.index)
    if key not in _checked:
        g = torch.Generator(device=device).manual_seed(0)
        a = torch.randn(384, 320, device=device, generator=g).to(torch.bfloat16)
        b = torch.randn(520, 320, device=device, generator=g).to(torch.bfloat16)
        ref = a.float() @ b.float().t()
        got = gemm_nt(a, b).float()
        _checked[key] = bool(((got - ref).abs().max() / ref.abs().max()).item() < 2e-2)
    return _checked[key]


def enabled() -> bool:
    return available() and _MODE in ("tcgen05", "auto")


def supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    if not enabled() or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.dim() != 2:
        return False
    if not _shape_ok(a, b):
        return False
    return _MODE == "tcgen05" or _self_check(a.device)


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if not supported(x2, w):
        return torch.nn.functional.linear(x, w, bias)
    y = _Linear.apply(x2, w)
    if bias is not None:
        y = y + bias
    return y.view(*shape[:-1], w.shape[0])
