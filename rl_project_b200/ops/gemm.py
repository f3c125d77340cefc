"""tcgen05/TMEM GEMMs (csrc/gemm_2sm.cu, csrc/gemm_tcgen05.cu) and the linear layer built on them.

One persistent warp-specialised kernel covers a linear layer's three GEMMs
without transposing anything:

* forward      ``y  = x  W^T``   A = x  [M, K] (K-major),   B = W [N, K] (K-major)
* input grad   ``dx = dy W``     A = dy [M, N] (K-major),   B = W stored [N, K] read MN-major
* weight grad  ``dW = dy^T x``   A = dy read MN-major,      B = x read MN-major

``RLB_GEMM`` selects the implementation of the model's plain linear layers:
``cublas`` (torch.matmul; the default), ``tcgen05`` (this library's kernels), ``auto``
(tcgen05 once the numerics self-check on the first call passed) or ``tuned``
(per product shape, the fastest of the 2-SM kernel with 256 x 256 tiles, with
256 x 512 tiles, and cuBLAS -- timed once with CUDA events on the first call of
that shape; accumulating and graph-captured calls keep the per-shape default) or
``hybrid`` (forward products on the 2-SM kernel, gradient products on cuBLAS).
``RLB_GEMM_KERNEL`` picks the kernel: ``2sm`` (default; CTA pairs issuing
``tcgen05.mma.cta_group::2`` on 256 x 256 tiles, TMA-store epilogue) or
``1sm`` (one CTA per 128 x 256 tile, register-to-global epilogue; the base of
the grouped and all-reduce variants).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from rl_project_b200.ops._ext import available, native

# plain dense layers default to cuBLAS: in the full 1B training step on B200 it measured 257-259 ms against
# 272-275 ms with the own kernel (per-shape benches are within a few percent either way; see the GEMM notes)
_MODE = os.environ.get("RLB_GEMM", "cublas")
_KERNEL = os.environ.get("RLB_GEMM_KERNEL", "2sm")
_NSUB = int(os.environ.get("RLB_GEMM_NSUB", "0"))  # 0: per shape; 1: 256 x 256 tiles; 2: 256 x 512 tiles
_checked: dict = {}


_CLUSTERS: dict = {}


def _pairs(device_index: int) -> int:
    if device_index not in _CLUSTERS:
        _CLUSTERS[device_index] = max(1, torch.cuda.get_device_properties(device_index).multi_processor_count // 2)
    return _CLUSTERS[device_index]


def nsub_for(M: int, N: int, epi: int, device_index: int = 0, a_mn: int = 0) -> int:
    """Tile width of the 2-SM kernel for a product.  256 x 512 tiles (one A slice feeds two MMAs: a quarter
    fewer operand bytes) unless the output is fp32, too narrow, A is read MN-major (the weight-gradient
    layout, measured faster with 256 x 256 tiles and their double-buffered accumulators: 1.02x against 0.89x
    of cuBLAS on the 1B model's 16384 x 2048 x 32768 weight gradient), or their last wave of CTA pairs would
    leave clearly more of the GPU idle than 256 x 256 tiles do."""
    if _NSUB:
        return _NSUB
    if epi != 0 or N <= 256 or a_mn:
        return 1
    pairs = _pairs(device_index)

    def wave_fill(bn: int) -> float:
        tiles = -(-M // 256) * -(-N // bn)
        waves = -(-tiles // pairs)
        return tiles / (waves * pairs)

    return 2 if wave_fill(512) + 0.05 >= wave_fill(256) else 1


def _describe(t: torch.Tensor) -> str:
    return (f"{tuple(t.shape)} stride {tuple(t.stride())} {t.dtype} {t.device} ptr%16={t.data_ptr() % 16} "
            f"contiguous={t.is_contiguous()}")


# ---------------------------------------------------------------- per-shape kernel choice ("tuned" mode)
# (a_mn, b_mn, epi, M, N, K, device) -> "own1" | "own2" | "cublas": the fastest of the 2-SM kernel with
# 256 x 256 tiles, with 256 x 512 tiles, and cuBLAS, timed with CUDA events on the first call of a shape
_TUNED: dict = {}
_TUNE_REPS = 3


def _launch(choice: str, a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha) -> None:
    if choice == "cublas":  # only offered for bf16 outputs, alpha 1 and a dense output
        lhs = a.t() if a_mn else a
        rhs = b if b_mn else b.t()
        torch.matmul(lhs, rhs, out=out)
        return
    native().gemm2(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, None, 0, 2 if choice == "own2" else 1)


def _candidates(epi: int, alpha: float, N: int, ldc: int):
    cands = ["own1"]
    if epi == 0 and N > 256:
        cands.append("own2")
    if epi == 0 and alpha == 1.0 and ldc == N:
        cands.append("cublas")
    return cands


def _choose(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha) -> str:
    key = (a_mn, b_mn, epi, M, N, K, a.device.index)
    got = _TUNED.get(key)
    if got is not None:
        return got
    default = "own2" if nsub_for(M, N, epi, a.device.index or 0, a_mn) == 2 else "own1"
    cands = _candidates(epi, alpha, N, ldc)
    if len(cands) == 1 or torch.cuda.is_current_stream_capturing() or epi != 0:
        return default  # accumulating outputs are never re-run; graphs cannot be timed
    times = {}
    for c in cands:
        _launch(c, a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)  # warm-up (and correct output)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(_TUNE_REPS):
            _launch(c, a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)
        t1.record()
        t1.synchronize()
        times[c] = t0.elapsed_time(t1)
    best = min(times, key=times.get)
    _TUNED[key] = best
    _launch(best, a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)
    return best


def tuned_choices() -> dict:
    """The kernel picked for every shape seen so far in ``tuned`` mode."""
    return dict(_TUNED)


def _run(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha):
    try:
        if _KERNEL == "1sm":
            native().gemm(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, None)
        elif _MODE == "tuned":
            key = (a_mn, b_mn, epi, M, N, K, a.device.index)
            if key in _TUNED:
                _launch(_TUNED[key], a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)
            else:
                choice = _choose(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)
                if key not in _TUNED:  # not timed (graph capture, accumulation): the per-shape default
                    _launch(choice, a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha)
        else:
            native().gemm2(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, None, 0,
                           nsub_for(M, N, epi, a.device.index or 0, a_mn))
    except RuntimeError as e:
        raise RuntimeError(f"{e} [a_mn={a_mn} b_mn={b_mn} epi={epi} M={M} N={N} K={K} lda={lda} ldb={ldb} "
                           f"ldc={ldc}; A {_describe(a)}; B {_describe(b)}; C {_describe(out)}; current device "
                           f"{torch.cuda.current_device()}]") from e


def _ok_ptr(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def _dense(t: torch.Tensor) -> torch.Tensor:
    """``t`` as a contiguous tensor whose base is 16-byte aligned (the TMA descriptors need both); a contiguous
    view at an odd storage offset -- e.g. a gradient slice handed over by autograd -- is copied."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def gemm_nt(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``a [M, K] @ b[N, K]^T`` in bf16 (fp32 accumulate)."""
    M, K = a.shape
    N = b.shape[0]
    a = _dense(a)
    b = _dense(b)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    _run(a, b, out, 0, 0, 0, M, N, K, K, K, out.stride(0), alpha)
    return out


def gemm_nn(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0) -> torch.Tensor:
    """``a [M, K] @ b [K, N]`` (b read MN-major, no transpose)."""
    M, K = a.shape
    N = b.shape[1]
    a = _dense(a)
    b = _dense(b)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    _run(a, b, out, 0, 1, 0, M, N, K, K, N, N, alpha)
    return out


def gemm_tn(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, out: Optional[torch.Tensor] = None,
            accumulate: bool = False) -> torch.Tensor:
    """``a [K, M]^T @ b [K, N]`` -> ``[M, N]`` (both read MN-major).  fp32 ``out`` + ``accumulate`` adds into it."""
    K, M = a.shape
    N = b.shape[1]
    a = _dense(a)
    b = _dense(b)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
        epi = 0
    else:
        epi = 2 if accumulate else (1 if out.dtype == torch.float32 else 0)
    _run(a, b, out, 1, 1, epi, M, N, K, M, N, out.stride(0), alpha)
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
        dy = _dense(dy)
        if not backward_own():  # "hybrid": the gradient products go to cuBLAS
            return (dy @ w if ctx.needs_input_grad[0] else None, dy.t() @ x2 if ctx.needs_input_grad[1] else None)
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
    return available() and _MODE in ("tcgen05", "auto", "tuned", "hybrid")


def backward_own() -> bool:
    """Whether the input- and weight-gradient products of the own linear layers run the own kernel too
    (every enabled mode except ``hybrid``, which keeps the forward on it and sends the gradients to cuBLAS)."""
    return enabled() and _MODE != "hybrid"


def supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    if not enabled() or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.dim() != 2:
        return False
    if not _shape_ok(a, b):
        return False
    return _MODE in ("tcgen05", "tuned", "hybrid") or _self_check(a.device)


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if not supported(x2, w):
        return torch.nn.functional.linear(x, w, bias)
    y = _Linear.apply(x2, w)
    if bias is not None:
        y = y + bias
    return y.view(*shape[:-1], w.shape[0])
