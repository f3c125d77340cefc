"""Row-parallel linear with the tensor-parallel all-reduce fused into the GEMM (comm path 3, forward).

The reference's ``RowParallelLinear`` runs the local GEMM and then an NCCL
``all_reduce`` of the whole output (``src/forgeline/distributed/tensor_parallel.py:18``),
which nothing overlaps.  Here the persistent tcgen05 GEMM (csrc/gemm_tcgen05.cu,
``rlb_gemm_allreduce``) finishes the reduction tile by tile inside its epilogue:

1. a tile's fp32 accumulator is rounded to bf16 and stored into this rank's
   partial buffer (the TMEM accumulator is released right away, so the next
   tile's MMAs start);
2. the tile's flag is raised in every rank's flag array (system-scope release);
3. after a bounded wait for every rank's flag of that tile, the epilogue sums
   all ranks' bf16 partials of the tile in rank order -- so every rank produces
   bit-identical output -- and stores the result.

Each rank computes tile t at the same point of its persistent schedule (same
shapes, same grid), so the exchange of one tile overlaps the MMAs of the next.
Partials and flags live in two slots of CUDA-IPC-shared buffers used on
alternate launches: a rank starts launch k + 2 (reusing slot k mod 2) only
after its launch k + 1 finished, which needed every peer's flags of launch
k + 1, which a peer raises only after its own launch k -- the last reader of
that slot -- finished.

The backward of the all-reduce is the identity, so the row-parallel layer's
backward is the ordinary local dgrad / wgrad.  The column-parallel layers that
open each block (q/k/v, w1/w3) have the mirror-image pattern: identity forward,
all-reduce of the input gradient backward.  ``column_parallel_linear_fused``
runs that backward as one GEMM (``dy @ W``, B operand stored [K][N]) with the
same epilogue all-reduce, instead of a local GEMM followed by an NCCL
all-reduce (``src/forgeline/distributed/tensor_parallel.py:39-70`` is the
reference's pair of collectives).  Forward and backward launches share the two
slots; every rank issues them in the same order (autograd's order is the same
on every rank of the group).
"""

from __future__ import annotations

import os
from typing import Any, Dict, Optional

import torch
import torch.distributed as dist

from rl_project_b200.core.errors import DistributedTimeoutError
from rl_project_b200.ops._ext import available, native
from rl_project_b200.observability.tracing import nvtx_annotate

BM, BN = 128, 256  # the GEMM's tile


def _tiles(M: int, N: int) -> int:
    return ((M + BM - 1) // BM) * ((N + BN - 1) // BN)


class GemmAllReduce:
    """Fused row-parallel GEMM + all-reduce for one tensor-parallel group (collective to construct)."""

    def __init__(self, group, max_elems: int, device: torch.device):
        from rl_project_b200.parallel.fused_comm import _IpcBuffers

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_elems = int(max_elems)
        self.max_tiles = self.max_elems // (BM * 32) + 4096  # N >= 32: bounds the tile count of any fitting call
        self.device = device
        self.mem = _IpcBuffers(group, 2 * self.max_elems * 2, 2 * self.max_tiles * self.world * 4, device)
        self.mem.flags_raw.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.grid = torch.cuda.get_device_properties(device).multi_processor_count
        self.launches = 0

    def fits(self, M: int, N: int) -> bool:
        return M * N <= self.max_elems and N % 32 == 0 and _tiles(M, N) <= self.max_tiles

    @nvtx_annotate("rlb/gemm_allreduce")
    def _launch(self, a: torch.Tensor, b: torch.Tensor, N: int, b_mn: int) -> torch.Tensor:
        slot = self.launches % 2
        epoch = self.launches // 2 + 1
        self.launches += 1
        part = [p + slot * self.max_elems * 2 for p in self.mem.buffer_ptrs]
        flag = [f + slot * self.max_tiles * self.world * 4 for f in self.mem.flag_ptrs]
        out = torch.empty(a.shape[0], N, dtype=torch.bfloat16, device=a.device)
        native().gemm_allreduce(a, b, out, part, flag, self.rank, epoch, 1.0, self.status, self.grid, b_mn)
        return out

    def __call__(self, x2: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``sum over ranks of x2 @ w^T`` (``w [N, K]``): the row-parallel output."""
        return self._launch(x2, w, w.shape[0], 0)

    def dgrad(self, g2: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``sum over ranks of g2 @ w`` (``w [N_local, C]``): the column-parallel input gradient."""
        return self._launch(g2, w, w.shape[1], 1)

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise DistributedTimeoutError(f"fused tensor-parallel all-reduce: a wait ran out (status 0x{code:x})",
                                          hint="A tensor-parallel rank stopped or fell behind.")

    def close(self) -> None:
        if self.mem is not None:
            self.mem.close()
            self.mem = None


_REDUCERS: Dict[Any, Optional[GemmAllReduce]] = {}
_ENABLED = os.environ.get("RLB_TP_FUSED", "1") != "0"


def set_enabled(flag: bool) -> None:
    """Strategy switch (``fused_comm`` off / nccl_baseline disables it)."""
    global _ENABLED
    _ENABLED = bool(flag)


def reducer_for(group, x2: torch.Tensor, N: int) -> Optional[GemmAllReduce]:
    """The fused reducer of ``group`` if this call can use it (same answer on every rank of the group)."""
    if not (_ENABLED and available() and x2.is_cuda and x2.dtype == torch.bfloat16 and dist.is_initialized()):
        return None
    if dist.get_backend(group) != "nccl" or dist.get_world_size(group) > 8:
        return None
    key = group if group is not None else "world"
    M = x2.shape[0]
    if key not in _REDUCERS:
        # sized for this first call with headroom; created collectively (every rank reaches the first call)
        _REDUCERS[key] = GemmAllReduce(group, max(M * N * 2, 1 << 22), x2.device)
    r = _REDUCERS[key]
    return r if r.fits(M, N) else None


def close_all() -> None:
    for r in _REDUCERS.values():
        if r is not None:
            r.close()
    _REDUCERS.clear()


class _RowParallelAR(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, w, reducer):
        ctx.save_for_backward(x2, w)
        return reducer(x2.contiguous(), w.contiguous())

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        g = g.contiguous()
        dx = g @ w if ctx.needs_input_grad[0] else None
        dw = g.t() @ x2 if ctx.needs_input_grad[1] else None
        return dx, dw, None


def row_parallel_linear_fused(x: torch.Tensor, w: torch.Tensor, reducer: GemmAllReduce) -> torch.Tensor:
    shape = x.shape
    y = _RowParallelAR.apply(x.reshape(-1, shape[-1]), w, reducer)
    return y.view(*shape[:-1], w.shape[0])


class _ColumnParallelAR(torch.autograd.Function):
    """Column-parallel linear whose input-gradient all-reduce is fused into the dgrad GEMM."""

    @staticmethod
    def forward(ctx, x2, w, reducer):
        from rl_project_b200.ops.linear import linear

        ctx.save_for_backward(x2, w)
        ctx.reducer = reducer
        return linear(x2, w)

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        g = g.contiguous()
        dx = ctx.reducer.dgrad(g, w.contiguous()) if ctx.needs_input_grad[0] else None
        dw = g.t() @ x2 if ctx.needs_input_grad[1] else None
        return dx, dw, None


def column_parallel_linear_fused(x: torch.Tensor, w: torch.Tensor, reducer: GemmAllReduce) -> torch.Tensor:
    """``x @ w^T`` for a row-split ``w [N_local, C]`` whose input ``x`` is replicated over the group:
    forward is the local GEMM; backward all-reduces ``dx`` inside the dgrad GEMM's epilogue."""
    shape = x.shape
    y = _ColumnParallelAR.apply(x.reshape(-1, shape[-1]), w, reducer)
    return y.view(*shape[:-1], w.shape[0])
