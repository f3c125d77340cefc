"""Grouped GEMMs for mixture-of-experts layers on the tcgen05 kernel (csrc/gemm_tcgen05.cu, grouped modes).

The reference runs every expert as its own ``nn.Linear`` calls inside a Python
loop over experts (``src/forgeline/models/moe/layer.py:32-38``).  Here one
launch covers all experts of a layer: the routed rows are laid out sorted by
expert with each expert's segment padded to a multiple of 128 rows (the
GEMM's M tile), so no tile mixes two experts, and a per-tile group table
tells the kernel which expert's weights a tile multiplies.  The buffer has a
static upper bound of rows (``rows_bound``) so building the layout needs no
host synchronisation; tiles past the used rows are skipped by the kernel.

* forward      ``y_e  = x_e W_e^T``   (M-grouped, W [E, N, K] read K-major)
* input grad   ``dx_e = dy_e W_e``    (M-grouped, W read MN-major; N % 64 == 0)
* weight grad  ``dW_e = dy_e^T x_e``  (K-grouped over each expert's rows)
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from rl_project_b200.ops._ext import native

ALIGN = 128  # rows per tile: every expert segment is padded to a multiple of this


def rows_bound(n_slots: int, n_groups: int) -> int:
    """Rows of the padded dispatch buffer for ``n_slots`` routed (token, expert) pairs over ``n_groups``."""
    r = n_slots + n_groups * (ALIGN - 1)
    return (r + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class GroupedLayout:
    rows: int                  # rows of the padded buffer (a multiple of ALIGN)
    dest: torch.Tensor         # [n_slots] int64: buffer row of each slot, slots in expert-sorted order
    tile_group: torch.Tensor   # [rows / ALIGN] int32: expert of each row tile, -1 past the used rows
    seg_start: torch.Tensor    # [E] int32: first row of each expert's segment
    seg_len: torch.Tensor      # [E] int32: padded rows of each expert's segment


def grouped_layout(sorted_experts: torch.Tensor, counts: torch.Tensor, rows: Optional[int] = None) -> GroupedLayout:
    """Layout of slots already sorted by expert (``sorted_experts`` [n_slots], ``counts`` [E]) on the device."""
    E = counts.numel()
    n = sorted_experts.numel()
    rows = rows if rows is not None else rows_bound(n, E)
    counts = counts.to(torch.int64)
    padded = (counts + ALIGN - 1) // ALIGN * ALIGN
    seg_end = torch.cumsum(padded, 0)
    seg_start = seg_end - padded
    cnt_start = torch.cumsum(counts, 0) - counts
    pos = torch.arange(n, device=counts.device)
    e = sorted_experts.to(torch.int64)
    dest = seg_start[e] + (pos - cnt_start[e])
    tile_start = torch.arange(rows // ALIGN, device=counts.device) * ALIGN
    owner = torch.searchsorted(seg_end, tile_start, right=True)
    tile_group = torch.where(tile_start < seg_end[-1], owner, torch.full_like(owner, -1)).to(torch.int32)
    return GroupedLayout(rows, dest, tile_group, seg_start.to(torch.int32), padded.to(torch.int32))


def grouped_nt(x: torch.Tensor, w: torch.Tensor, tile_group: torch.Tensor) -> torch.Tensor:
    """``x [R, K]`` rows of expert e times ``w[e] [N, K]^T`` -> ``[R, N]`` (rows of skipped tiles undefined)."""
    R, K = x.shape
    E, N, K2 = w.shape
    assert K == K2
    out = torch.empty(R, N, dtype=torch.bfloat16, device=x.device)
    native().gemm_grouped(1, 0, 0, x, w, out, R, N, K, K, K, N, 1.0, E, tile_group, None, None, 0, None)
    return out


def grouped_nn(dy: torch.Tensor, w: torch.Tensor, tile_group: torch.Tensor) -> torch.Tensor:
    """``dy [R, N]`` rows of expert e times ``w[e] [N, K]`` -> ``[R, K]`` (N must be a multiple of 64)."""
    R, N = dy.shape
    E, N2, K = w.shape
    assert N == N2 and N % 64 == 0
    out = torch.empty(R, K, dtype=torch.bfloat16, device=dy.device)
    native().gemm_grouped(1, 1, 0, dy, w, out, R, K, N, N, K, K, 1.0, E, tile_group, None, None, 0, None)
    return out


def grouped_tn(dy: torch.Tensor, x: torch.Tensor, seg_start: torch.Tensor, seg_len: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per expert e: ``dy[seg]^T x[seg]`` -> ``[E, N, K]`` (zero for experts without rows)."""
    R, N = dy.shape
    R2, K = x.shape
    assert R == R2
    E = seg_start.numel()
    if out is None:
        out = torch.empty(E, N, K, dtype=torch.bfloat16, device=dy.device)
    assert out.shape == (E, N, K) and out.is_contiguous() and out.dtype == torch.bfloat16
    native().gemm_grouped(2, 1, 0, dy, x, out, N, K, R, N, K, K, 1.0, E, None, seg_start, seg_len, R, None)
    return out


class _GroupedSwiGLU(torch.autograd.Function):
    """SwiGLU experts over a padded grouped layout: ``y = (silu(x W1^T) * (x W3^T)) W2^T`` per expert.

    Inputs: the padded rows ``xp [R, C]``, the layout, the stacked ``w13 [E, 2F, C]`` / ``w2 [E, C, F]``, a
    gradient ``sink`` and the per-expert parameters the stacked weights hold, ordered
    ``[w1_0..w1_{E-1}, w3_0.., w2_0..]``.  With a sink the weight gradients are written by the grouped kernel
    straight into two packed buffers kept in the sink, and each parameter's ``.grad`` is a view into them
    (accumulated in place on later micro-batches) -- no per-expert copies.  Without parameters the stacked
    weights came from differentiable ops and receive the gradients themselves."""

    @staticmethod
    def forward(ctx, xp, tile_group, seg_start, seg_len, w13, w2, sink, *params):
        C = native()
        h13 = grouped_nt(xp, w13, tile_group)
        a = C.swiglu_fwd(h13)
        y = grouped_nt(a, w2, tile_group)
        ctx.save_for_backward(xp, tile_group, seg_start, seg_len, w13, w2, h13, a)
        ctx.sink = sink
        ctx.params = params
        return y

    @staticmethod
    def backward(ctx, dy):
        C = native()
        xp, tile_group, seg_start, seg_len, w13, w2, h13, a = ctx.saved_tensors
        dy = dy.contiguous()
        da = grouped_nn(dy, w2, tile_group)
        dh13 = C.swiglu_bwd(h13, da)
        dxp = grouped_nn(dh13, w13, tile_group) if ctx.needs_input_grad[0] else None
        ps = ctx.params
        if not ps:  # stacked weights built from the parameters by differentiable ops
            return (dxp, None, None, None, grouped_tn(dh13, xp, seg_start, seg_len),
                    grouped_tn(dy, a, seg_start, seg_len), None)
        E, F = w13.shape[0], w2.shape[2]
        sink = ctx.sink
        g13, g2 = sink.get("g13"), sink.get("g2")
        if g13 is None:
            g13, g2 = torch.empty_like(w13), torch.empty_like(w2)
            sink["g13"], sink["g2"] = g13, g2
        views = [g13[e, :F] for e in range(E)] + [g13[e, F:] for e in range(E)] + [g2[e] for e in range(E)]
        if all(p.grad is None for p in ps):
            grouped_tn(dh13, xp, seg_start, seg_len, out=g13)
            grouped_tn(dy, a, seg_start, seg_len, out=g2)
            for p, v in zip(ps, views):
                p.grad = v
        elif all(p.grad is not None and p.grad.data_ptr() == v.data_ptr() for p, v in zip(ps, views)):
            g13.add_(grouped_tn(dh13, xp, seg_start, seg_len))
            g2.add_(grouped_tn(dy, a, seg_start, seg_len))
        else:  # gradients rebound elsewhere: accumulate parameter by parameter
            d13, d2 = grouped_tn(dh13, xp, seg_start, seg_len), grouped_tn(dy, a, seg_start, seg_len)
            new = [d13[e, :F] for e in range(E)] + [d13[e, F:] for e in range(E)] + [d2[e] for e in range(E)]
            for p, d in zip(ps, new):
                p.grad = d.clone() if p.grad is None else p.grad.add_(d)
        return (dxp, None, None, None, None, None, None) + (None,) * len(ps)


def grouped_swiglu_experts(xp, layout: GroupedLayout, w13, w2, params=(), sink=None):
    return _GroupedSwiGLU.apply(xp, layout.tile_group, layout.seg_start, layout.seg_len, w13, w2,
                                sink if sink is not None else {}, *params)
