"""tcgen05/TMEM GEMMs (csrc/gemm_2sm.cu, csrc/gemm_tcgen05.cu) and the linear layer built on them.

One persistent warp-specialised kernel covers a linear layer's three GEMMs
without transposing anything:

* forward      ``y  = x  W^T``   A = x  [M, K] (K-major),   B = W [N, K] (K-major)
* input grad   ``dx = dy W``     A = dy [M, N] (K-major),   B = W stored [N, K] read MN-major
* weight grad  ``dW = dy^T x``   A = dy read MN-major,      B = x read MN-major

``RLB_GEMM`` selects the implementation of the model's plain linear layers:
``cublas`` (torch.matmul), ``tcgen05`` (this library's kernels), ``auto``
(tcgen05 once the numerics self-check on the first call passed) or ``tuned``
(per product shape, the fastest of the 2-SM kernel with 256 x 256 tiles, with
256 x 512 tiles, and cuBLAS -- timed once with CUDA events on the first call of
that shape; accumulating and graph-captured calls keep the per-shape default) or
``hybrid`` (the default: forward products on the 2-SM kernel, with fused epilogues where one applies --
the gated FFN's projection with the SwiGLU activation, the attention projection with RoPE and the q / k / v
split, the LM head with per-row log-sum-exp statistics -- and gradient products on cuBLAS) or ``fwd_dgrad``
(forward and input-gradient products on the 2-SM kernel, weight gradients on cuBLAS).  Products too small to
give every CTA pair a tile (decode steps, short prefills) go to cuBLAS in every mode (``fills_gpu``).
``RLB_GEMM_KERNEL`` picks the kernel: ``2sm`` (default; CTA pairs issuing
``tcgen05.mma.cta_group::2`` on 256 x 256 or 256 x 512 tiles, TMA-store epilogue) or
``1sm`` (one CTA per 128 x 256 tile, register-to-global epilogue; the base of
the grouped and all-reduce variants).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from rl_project_b200.ops._ext import available, native

# default "hybrid": in the full 1B training step on B200 (alternating runs on one box) the own forward products
# with the fused epilogues and cuBLAS gradients measured 256.5-257.0 ms against 257.9-258.8 ms for all-cuBLAS;
# own input- and weight-gradient products still cost 1.5-4 % in the step under the power cap
_MODE = os.environ.get("RLB_GEMM", "hybrid")
_KERNEL = os.environ.get("RLB_GEMM_KERNEL", "2sm")
_NSUB = int(os.environ.get("RLB_GEMM_NSUB", "0"))  # 0: per shape; 1: 256 x 256 tiles; 2: 256 x 512 tiles
_GROUP_M = int(os.environ.get("RLB_GEMM_GROUP_M", "0"))  # raster group height in M tiles (0: kernel default)
_SPLITK = os.environ.get("RLB_GEMM_SPLITK", "auto")  # "auto" | "off" | a fixed split count
_MIN_TILES = int(os.environ.get("RLB_GEMM_MIN_TILES", "-1"))  # layers' own-kernel threshold (-1: one per CTA pair)
_MAX_CTAS = int(os.environ.get("RLB_GEMM_MAX_CTAS", "0"))  # cap on the persistent grid (0: every SM)
# gated FFN backward: "1" runs the down projection's input gradient with the SwiGLU backward in its epilogue.
# Off by default: its epilogue reads gate and up with per-thread global loads (each lane a different row), which
# are latency-bound -- 3.43 ms against 0.68 ms cuBLAS + 0.43 ms activation backward at 32768 x 8192 x 2048 on
# B200; staging those tiles through shared memory with TMA is what it would need
_SWIGLU_BWD = os.environ.get("RLB_GEMM_SWIGLU_BWD", "0") == "1"
_checked: dict = {}


_CLUSTERS: dict = {}


def _pairs(device_index: int) -> int:
    if device_index not in _CLUSTERS:
        _CLUSTERS[device_index] = max(1, torch.cuda.get_device_properties(device_index).multi_processor_count // 2)
    return _CLUSTERS[device_index]


def nsub_for(M: int, N: int, epi: int, device_index: int = 0, a_mn: int = 0) -> int:
    """Tile width of the 2-SM kernel for a product.  256 x 512 tiles (one A slice feeds two MMAs: a quarter
    fewer operand bytes per FLOP, which under the 1 kW power cap is a higher sustained clock) unless the output
    is fp32 or too narrow.  Weight gradients (A read MN-major, long K) always take them: their wave
    quantisation is evened out by splitting K (``k_splits``); sustained on B200 this measured 0.92-1.00x of
    cuBLAS against 0.75-0.94x with 256 x 256 tiles on the 1B model's weight gradients.  For the other
    layouts, 256 x 256 tiles when the last wave of 256 x 512 tiles would leave clearly more of the GPU idle."""
    if _NSUB:
        return _NSUB
    if epi != 0 or N <= 256:
        return 1
    if a_mn:
        return 2
    pairs = _pairs(device_index)

    def wave_fill(bn: int) -> float:
        tiles = -(-M // 256) * -(-N // bn)
        waves = -(-tiles // pairs)
        return tiles / (waves * pairs)

    return 2 if wave_fill(512) + 0.05 >= wave_fill(256) else 1


def group_for(N: int, a_mn: int) -> int:
    """Raster group height (M tiles walked before moving to the next N tile).  Wide outputs (N >= 8192: the
    w1|w3 and LM-head forward, the w2 input gradient) walk 32 M tiles, so each B tile is read by all the CTA
    pairs that need it while it is in L2 instead of being re-read from HBM for every group of 8; measured
    under the power cap on B200 this lifted the LM-head forward from 0.96x to 1.00x of cuBLAS (and its SM
    clock from 1267 to 1305 MHz).  Narrower outputs and weight gradients keep groups of 8."""
    if _GROUP_M:
        return _GROUP_M
    return 32 if (N >= 8192 and not a_mn) else 8


# per-unit cost of a K-split work unit beyond its MMAs (pipeline fill, accumulator drain), in 64-deep K slices
_UNIT_OVERHEAD = 4.0


def k_splits(M: int, N: int, K: int, nsub: int, device_index: int = 0) -> int:
    """K ranges per output tile for a weight-gradient product (bf16 output): more than one when the tiles
    alone would leave much of the last wave of CTA pairs idle and K is long enough to divide -- e.g. the
    1B model's q|k|v weight gradient (3072 x 2048 over K = 32768: 96 tiles for 74 CTA pairs, two waves at
    65 % occupancy) runs as three ranges of 170 K slices (288 units, 3.9 waves).  The model counts a unit as
    its K slices plus a fixed overhead, and a split must save 6 % of it to pay for the fp32 partial sums'
    zero fill and the final bf16 conversion."""
    if _SPLITK == "off":
        return 1
    nk = -(-K // 64)
    if _SPLITK != "auto":
        return max(1, min(int(_SPLITK), nk))
    pairs = _pairs(device_index)
    tiles = -(-M // 256) * -(-N // (256 * nsub))

    def cost(sp: int) -> float:
        return -(-tiles * sp // pairs) * (nk / sp + _UNIT_OVERHEAD)

    best = min((sp for sp in range(1, 9) if sp == 1 or nk // sp >= 16), key=cost)
    return best if cost(best) < 0.94 * cost(1) else 1


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
    native().gemm2x(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, None, _MAX_CTAS, 2 if choice == "own2" else 1,
                    1, group_for(N, a_mn))


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
            nsub = nsub_for(M, N, epi, a.device.index or 0, a_mn)
            splits = k_splits(M, N, K, nsub, a.device.index or 0) if (a_mn and epi == 0) else 1
            if splits > 1:  # partial products reduce-added into fp32, then rounded once to bf16
                acc = torch.zeros(M, N, dtype=torch.float32, device=a.device)
                native().gemm2x(a, b, acc, a_mn, b_mn, 2, M, N, K, lda, ldb, N, alpha, None, _MAX_CTAS, nsub, splits,
                                group_for(N, a_mn))
                out.copy_(acc)
            else:
                native().gemm2x(a, b, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, None, _MAX_CTAS, nsub, 1,
                                group_for(N, a_mn))
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
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dy, w) if dgrad_own() else dy @ w
        if ctx.needs_input_grad[1]:
            dw = gemm_tn(dy, x2) if wgrad_own() else dy.t() @ x2
        return dx, dw


def gemm_nt_swiglu(x2: torch.Tensor, w13: torch.Tensor):
    """``h13 = x2 w13^T`` for ``w13 = [W1; W3]`` and ``act = silu(h13[:, :H]) * h13[:, H:]`` from one GEMM whose
    epilogue applies the activation (256 x 512 tiles pairing the gate and up columns of 256 hidden units)."""
    x2, w13 = _dense(x2), _dense(w13)
    M, H = x2.shape[0], w13.shape[0] // 2
    h13 = torch.empty(M, 2 * H, dtype=torch.bfloat16, device=x2.device)
    act = torch.empty(M, H, dtype=torch.bfloat16, device=x2.device)
    native().gemm2_swiglu(x2, w13, h13, act, group_for(2 * H, 0), _MAX_CTAS)
    return h13, act


class _LinearSwiGLU(torch.autograd.Function):
    """Gated FFN input projection + activation: forward in one GEMM (activation in its epilogue); backward
    through the activation kernel and the linear layer's two gradient products."""

    @staticmethod
    def forward(ctx, x2, w13):
        h13, act = gemm_nt_swiglu(x2, w13)
        ctx.save_for_backward(x2, w13, h13)
        return act

    @staticmethod
    def backward(ctx, da):
        x2, w13, h13 = ctx.saved_tensors
        dh13 = native().swiglu_bwd(h13, _dense(da))
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dh13, w13) if dgrad_own() else dh13 @ w13
        if ctx.needs_input_grad[1]:
            dw = gemm_tn(dh13, x2) if wgrad_own() else dh13.t() @ x2
        return dx, dw


def gemm_dgrad_swiglu(dy: torch.Tensor, w2: torch.Tensor, h13: torch.Tensor) -> torch.Tensor:
    """``dh13`` = SwiGLU backward of ``dy w2`` against ``h13`` in one GEMM (``w2 [d, H]``, the down projection's
    weight): the activation's input gradient without storing ``dy w2``."""
    dy, w2 = _dense(dy), _dense(w2)
    dh13 = torch.empty(dy.shape[0], 2 * w2.shape[1], dtype=torch.bfloat16, device=dy.device)
    native().gemm2_dgrad_swiglu(dy, w2, h13, dh13, group_for(w2.shape[1], 0), _MAX_CTAS)
    return dh13


class _SwiGLUFFN(torch.autograd.Function):
    """A whole gated FFN, ``out = (silu(x W1^T) * (x W3^T)) W2^T``, on the own GEMM's fused epilogues: forward
    projection + activation in one GEMM; backward, the down projection's input gradient + the activation's
    backward in one GEMM; the other products as the mode selects."""

    @staticmethod
    def forward(ctx, x2, w13, w2):
        h13, act = gemm_nt_swiglu(x2, w13)
        out = gemm_nt(act, w2) if supported(act, w2) else act @ w2.t()
        ctx.save_for_backward(x2, w13, w2, h13, act)
        return out

    @staticmethod
    def backward(ctx, dout):
        x2, w13, w2, h13, act = ctx.saved_tensors
        dout = _dense(dout)
        if _SWIGLU_BWD:
            dh13 = gemm_dgrad_swiglu(dout, w2, h13)
        else:
            da = gemm_nn(dout, w2) if dgrad_own() else dout @ w2
            dh13 = native().swiglu_bwd(h13, da)
        dw2 = (gemm_tn(dout, act) if wgrad_own() else dout.t() @ act) if ctx.needs_input_grad[2] else None
        dx = (gemm_nn(dh13, w13) if dgrad_own() else dh13 @ w13) if ctx.needs_input_grad[0] else None
        dw13 = (gemm_tn(dh13, x2) if wgrad_own() else dh13.t() @ x2) if ctx.needs_input_grad[1] else None
        return dx, dw13, dw2


def swiglu_ffn(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """Gated FFN on the fused GEMM epilogues (``w13 = [W1; W3]``, ``w2 [d, H]``)."""
    shape = x.shape
    out = _SwiGLUFFN.apply(x.reshape(-1, shape[-1]), w13, w2)
    return out.view(*shape[:-1], w2.shape[0])


def swiglu_fusable(x2: torch.Tensor, w13: torch.Tensor) -> bool:
    return (enabled() and _MODE != "tuned" and x2.dtype == torch.bfloat16 and w13.dtype == torch.bfloat16
            and x2.dim() == 2 and x2.shape[0] > 0 and (w13.shape[0] // 2) % 8 == 0 and w13.shape[0] % 2 == 0
            and x2.shape[1] % 8 == 0 and _ok_ptr(x2) and _ok_ptr(w13)
            and fills_gpu(x2.shape[0], w13.shape[0] // 2, 256, x2.device.index or 0))


def linear_swiglu(x: torch.Tensor, w13: torch.Tensor) -> torch.Tensor:
    """``silu(x W1^T) * (x W3^T)`` for ``w13 = [W1; W3]``; the activation is fused into the GEMM epilogue."""
    shape = x.shape
    act = _LinearSwiGLU.apply(x.reshape(-1, shape[-1]), w13)
    return act.view(*shape[:-1], w13.shape[0] // 2)


# rows from which the LM-head forward takes the log-sum-exp epilogue: measured on B200 (CUDA events, L2 flushed)
# 1.08x faster than GEMM + log-softmax pass at 32768 x 128256 x 2048, but 0.83x at 4096 x 32768 x 2048
_LSE_MIN_ROWS = int(os.environ.get("RLB_GEMM_LSE_MIN_ROWS", "16384"))


def lse_fusable(h: torch.Tensor, w: torch.Tensor) -> bool:
    """Whether the LM-head forward ``h W^T`` takes the GEMM whose epilogue also writes the rows' log-sum-exp
    statistics (the own kernel handles the forward in the current mode, the product fills the GPU, and there
    are enough rows for the fusion to pay)."""
    return h.shape[0] >= _LSE_MIN_ROWS and supported(h, w) and w.shape[0] >= 512


def gemm_nt_lse(h: torch.Tensor, w: torch.Tensor):
    """``logits = h w^T`` (bf16) plus, per row and per 256-column half tile, ``(max, sum exp(x - max),
    sum exp(x - max) x)`` of the stored bf16 logits: ``stats [M, 2 * ceil(N / 512), 4]`` fp32."""
    h, w = _dense(h), _dense(w)
    M, N = h.shape[0], w.shape[0]
    logits = torch.empty(M, N, dtype=torch.bfloat16, device=h.device)
    stats = torch.empty(M, 2 * (-(-N // 512)), 4, dtype=torch.float32, device=h.device)
    native().gemm2_lse(h, w, logits, stats, group_for(N, 0), _MAX_CTAS)
    return logits, stats


def rope_qkv_fusable(x2: torch.Tensor, w: torch.Tensor, n_head: int, n_kv_head: int, head_dim: int) -> bool:
    """Whether the attention input projection can run as one GEMM with RoPE and the q / k / v split in its
    epilogue (own kernel on the forward, head dim 64 or 128, whole 128-column blocks per q / k / v range)."""
    return (head_dim in (64, 128) and (n_head * head_dim) % 128 == 0 and (n_kv_head * head_dim) % 128 == 0
            and supported(x2, w))


class _LinearRopeQKV(torch.autograd.Function):
    """q, k, v = rope(split(x w^T)): forward in one GEMM; backward through the RoPE kernel's inverse rotation
    (which re-interleaves dq | dk | dv) and the linear layer's two gradient products."""

    @staticmethod
    def forward(ctx, x2, w, cos, sin, positions, B, T, Hq, Hkv, D, offset):
        x2, w = _dense(x2), _dense(w)
        q, k, v = native().gemm2_rope_qkv(x2, w, cos, sin, positions, B, T, Hq, Hkv, D, offset, group_for(w.shape[0], 0),
                                          _MAX_CTAS)
        ctx.save_for_backward(x2, w, cos, sin, positions if positions is not None else torch.empty(0))
        ctx.args = (B, T, Hq, Hkv, D, offset, positions is not None)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2, w, cos, sin, pos = ctx.saved_tensors
        B, T, Hq, Hkv, D, offset, has_pos = ctx.args
        dq = torch.zeros((B, T, Hq, D), dtype=x2.dtype, device=x2.device) if dq is None else dq.contiguous()
        dk = torch.zeros((B, T, Hkv, D), dtype=x2.dtype, device=x2.device) if dk is None else dk.contiguous()
        dv = torch.zeros((B, T, Hkv, D), dtype=x2.dtype, device=x2.device) if dv is None else dv.contiguous()
        dy = native().rope_qkv_bwd(dq, dk, dv, cos, sin, pos if has_pos else None, B, T, Hq, Hkv, D, offset,
                                   False).view(B * T, -1)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dy, w) if dgrad_own() else dy @ w
        if ctx.needs_input_grad[1]:
            dw = gemm_tn(dy, x2) if wgrad_own() else dy.t() @ x2
        return dx, dw, None, None, None, None, None, None, None, None, None


def linear_rope_qkv(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                    positions: Optional[torch.Tensor], n_head: int, n_kv_head: int, head_dim: int, offset: int = 0):
    """``x [B, T, C]`` -> token-major ``q [B, T, Hq, D]``, ``k``, ``v [B, T, Hkv, D]`` with RoPE applied to q and
    k inside the projection GEMM's epilogue (cos / sin tables ``[rows, D/2]`` fp32 on the device)."""
    B, T, C = x.shape
    pos = positions.to(torch.int32).reshape(-1).contiguous() if positions is not None else None
    return _LinearRopeQKV.apply(x.reshape(B * T, C), w, cos, sin, pos, B, T, n_head, n_kv_head, head_dim, offset)


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
    return available() and _MODE in ("tcgen05", "auto", "tuned", "hybrid", "fwd_dgrad")


def dgrad_own() -> bool:
    """Whether input-gradient products (``dy W``) run the own kernel: every enabled mode except ``hybrid``."""
    return enabled() and _MODE != "hybrid"


def wgrad_own() -> bool:
    """Whether weight-gradient products (``dy^T x``) run the own kernel: not under ``hybrid`` (all gradient
    products on cuBLAS) nor ``fwd_dgrad`` (forward and input gradients on the own kernel, weight gradients --
    the MN-major x MN-major layout where it is furthest behind cuBLAS under the power cap -- on cuBLAS)."""
    return enabled() and _MODE not in ("hybrid", "fwd_dgrad")


def backward_own() -> bool:
    """Whether every gradient product runs the own kernel."""
    return dgrad_own() and wgrad_own()


def fills_gpu(M: int, N: int, tile_n: int, device_index: int = 0) -> bool:
    """Whether a product has at least one 256 x ``tile_n`` output tile per CTA pair (``RLB_GEMM_MIN_TILES``
    overrides the count).  Smaller products -- decode steps, short prefills -- would leave most of the GPU
    idle on the persistent 2-SM kernel, so the layers send them to cuBLAS."""
    need = _MIN_TILES if _MIN_TILES >= 0 else _pairs(device_index)
    return -(-M // 256) * -(-N // tile_n) >= need


def supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    if not enabled() or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.dim() != 2:
        return False
    if not _shape_ok(a, b) or not fills_gpu(a.shape[0], b.shape[0], 512, a.device.index or 0):
        return False
    return _MODE in ("tcgen05", "tuned", "hybrid", "fwd_dgrad") or _self_check(a.device)


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if not supported(x2, w):
        return torch.nn.functional.linear(x, w, bias)
    y = _Linear.apply(x2, w)
    if bias is not None:
        y = y + bias
    return y.view(*shape[:-1], w.shape[0])
