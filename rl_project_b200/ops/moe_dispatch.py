"""Atomic-free dispatch and combine between token order and the padded
expert-sorted buffer of the grouped expert GEMMs (ops/grouped_gemm.py).

The reference's MoE scatters expert outputs back with masked in-place adds
(``src/forgeline/models/moe/layer.py:32-38``); a scatter-add with repeated
token indices (``index_add_``) is an atomic read-modify-write per element.
Here both directions of both operations are gathers:

* dispatch  ``xp[r] = x[token_of_row[r]]`` (padding rows read a zero row);
  its gradient ``dx[t] = sum_j dxp[row_of_slot[t, j]]`` is a gather of the
  ``k`` rows of each token followed by a dense sum over ``k``;
* combine   ``out[t] = sum_j w[t, j] y[row_of_slot[t, j]]``; its gradient
  with respect to ``y`` is a gather through ``slot_of_row`` (each buffer row
  holds at most one slot) and with respect to ``w`` a row-wise dot product.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class RowMaps:
    rows: int
    k: int
    row_of_slot: torch.Tensor  # [N*k] buffer row of each (token, j) slot
    slot_of_row: torch.Tensor  # [rows] slot held by each buffer row, N*k for padding rows
    token_of_row: torch.Tensor  # [rows] token of each buffer row, N for padding rows


def row_maps(order: torch.Tensor, dest: torch.Tensor, rows: int, k: int) -> RowMaps:
    """``order`` [N*k]: original slot of each expert-sorted position; ``dest`` [N*k]: buffer row of each
    sorted position (from grouped_layout)."""
    n_slots = order.numel()
    slot_of_row = torch.full((rows,), n_slots, dtype=torch.int64, device=order.device)
    slot_of_row[dest] = order
    row_of_slot = torch.empty(n_slots, dtype=torch.int64, device=order.device)
    row_of_slot[order] = dest
    return RowMaps(rows, k, row_of_slot, slot_of_row, torch.div(slot_of_row, k, rounding_mode="floor"))


def _acc_dtype(dt: torch.dtype) -> torch.dtype:
    """fp32 accumulation for 16-bit rows, the rows' own precision otherwise."""
    return torch.float32 if dt in (torch.bfloat16, torch.float16) else dt


def _with_zero_row(x: torch.Tensor) -> torch.Tensor:
    return torch.cat([x, x.new_zeros(1, x.shape[1])], 0)


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, maps: RowMaps):
        ctx.maps = maps
        ctx.n = x.shape[0]
        return _with_zero_row(x).index_select(0, maps.token_of_row)

    @staticmethod
    def backward(ctx, dxp):
        m = ctx.maps
        dx = dxp.index_select(0, m.row_of_slot).view(ctx.n, m.k, dxp.shape[1]).sum(1)
        return dx, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w, maps: RowMaps):
        n = w.shape[0]
        ys = y.index_select(0, maps.row_of_slot).view(n, maps.k, y.shape[1])
        ctx.save_for_backward(ys, w)
        ctx.maps = maps
        acc = _acc_dtype(y.dtype)
        return (ys.to(acc) * w.unsqueeze(-1).to(acc)).sum(1).to(y.dtype)

    @staticmethod
    def backward(ctx, dout):
        ys, w = ctx.saved_tensors
        m = ctx.maps
        n, k = w.shape
        acc = _acc_dtype(ys.dtype)
        dw = (ys.to(acc) * dout.to(acc).unsqueeze(1)).sum(-1).to(w.dtype) if ctx.needs_input_grad[1] else None
        dy = None
        if ctx.needs_input_grad[0]:
            dslot = (dout.unsqueeze(1) * w.unsqueeze(-1).to(dout.dtype)).reshape(n * k, -1)
            dy = _with_zero_row(dslot).index_select(0, m.slot_of_row)
        return dy, dw, None


def dispatch(x: torch.Tensor, maps: RowMaps) -> torch.Tensor:
    """``x [N, C]`` token rows -> ``[rows, C]`` padded expert-sorted buffer (each token in its k rows)."""
    return _Dispatch.apply(x, maps)


def combine(y: torch.Tensor, w: torch.Tensor, maps: RowMaps) -> torch.Tensor:
    """Expert outputs ``y [rows, C]`` and routing weights ``w [N, k]`` -> ``[N, C]``."""
    return _Combine.apply(y, w, maps)
