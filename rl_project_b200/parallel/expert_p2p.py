"""Expert-parallel dispatch and combine over NVLink peer memory (comm path 4).

The reference has no expert parallelism: every rank holds every expert and
dispatch is a Python mask loop (``src/forgeline/models/moe/layer.py:32-38``).
This framework's NCCL path (parallel/expert.py) exchanges counts, synchronises the host for
split sizes, runs ``all_to_all_single`` twice per layer and pass, and
re-permutes the received rows by expert on both sides.  Here every exchange is
one pull:

* each rank packs the rows it offers (its routed rows sorted by expert, or
  the expert outputs of its own padded layout) into its slot of an
  :class:`ExchangeRing` (a CUDA-IPC buffer mapped on every rank of the group)
  and raises its flag for the slot on every rank;
* after a one-thread bounded wait for every peer's flag, one gather kernel
  (csrc/comm_fused.cu ``gather_rows``) pulls exactly the rows this rank needs
  straight out of the peers' slots into their final place: the expert owner
  pulls its tokens directly into the padded expert-sorted layout of the
  grouped expert GEMMs (rl_project_b200/ops/grouped_gemm.py), and the token
  owner pulls its results directly into expert-sorted slot order.

Two row maps describe a layer: the dispatch map (each row of this rank's
padded layout <- (source rank, row of its packed rows)) and the combine map
(each of this rank's slots <- (expert owner, row of its layout)); the backward
of dispatch is a pull through the combine map and vice versa.  They are built
on the host from the all-gathered per-expert counts (one small synchronisation
per layer, as the NCCL path's split sizes need).

Slot reuse: every exchange packs, signals, waits and pulls on the current
stream, so a rank packs sequence ``q`` only after its own pull of ``q - 1``
finished; that pull needed every peer's signal ``q - 1``, which a peer raises
only after its pull of ``q - 2`` -- the last read of any slot it could still be
reading -- finished.  Four slots leave margin.
"""

from __future__ import annotations

import os
from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from rl_project_b200.core.errors import DistributedTimeoutError
from rl_project_b200.ops._ext import available, native
from rl_project_b200.observability.tracing import nvtx_annotate

NSLOTS = 4
ALIGN = 128  # the grouped GEMM's M tile: expert segments are padded to it


class ExchangeRing:
    """A ring of peer-visible row buffers ``[slot_rows, C]`` bf16 plus flags for one process group."""

    def __init__(self, group, slot_rows: int, C: int, device: torch.device, timeout_s: float = 120.0):
        from rl_project_b200.parallel.fused_comm import _IpcBuffers

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slot_rows, self.C = int(slot_rows), int(C)
        self.device = device
        self.mem = _IpcBuffers(group, NSLOTS * self.slot_rows * self.C * 2, NSLOTS * self.world * 4, device)
        self.buf = self.mem.buf_raw.view(torch.bfloat16).view(NSLOTS, self.slot_rows, self.C)
        self.flags = self.mem.flags_raw.view(torch.int32)
        self.flags.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        slot_bytes = self.slot_rows * self.C * 2
        self.bases = torch.tensor([[b + s * slot_bytes for b in self.mem.buffer_ptrs] for s in range(NSLOTS)],
                                  dtype=torch.int64, device=device)
        self.flag_ptrs = torch.tensor(self.mem.flag_ptrs, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.limit_ns = int(timeout_s * 1e9)
        self.seq = 0

    @nvtx_annotate("rlb/ep_exchange")
    def exchange(self, local: torch.Tensor, src_rank: torch.Tensor, src_row: torch.Tensor) -> torch.Tensor:
        """Offer ``local`` [n, C] to the group and return rows ``(src_rank[i], src_row[i])`` of the ranks' offers."""
        C = native()
        q = self.seq
        s, epoch = q % NSLOTS, q // NSLOTS + 1
        self.seq += 1
        n = local.shape[0]
        if n:
            self.buf[s, :n].copy_(local)
        C.signal_peers(self.flag_ptrs, self.rank, s, epoch)
        C.wait_peers(self.flags, self.world, s, epoch, self.limit_ns, self.status)
        out = torch.empty(src_rank.numel(), self.C, dtype=torch.bfloat16, device=self.device)
        C.gather_rows(self.bases[s], src_rank, src_row, out, self.slot_rows, self.status)
        return out

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise DistributedTimeoutError(f"expert-parallel exchange failed (status 0x{code:x})",
                                          hint="An expert-parallel rank stopped or fell behind.")

    def close(self) -> None:
        if self.mem is not None:
            self.mem.close()
            self.mem = None


class _Exchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local, ring, fwd_rank, fwd_row, bwd_rank, bwd_row):
        ctx.ring = ring
        ctx.save_for_backward(bwd_rank, bwd_row)
        return ring.exchange(local.contiguous(), fwd_rank, fwd_row)

    @staticmethod
    def backward(ctx, g):
        bwd_rank, bwd_row = ctx.saved_tensors
        return ctx.ring.exchange(g.contiguous(), bwd_rank, bwd_row), None, None, None, None, None


def _excl_cumsum(a: np.ndarray, axis: int = -1) -> np.ndarray:
    return np.cumsum(a, axis=axis) - a


def build_maps(cnt_all: np.ndarray, me: int, El: int) -> Dict[str, np.ndarray]:
    """Row maps of one layer from the all-gathered counts ``cnt_all [world, E]`` (slots per source and expert).

    Returns int32 arrays: dispatch ``d_rank, d_row`` (this rank's padded layout, -1 for padding), combine
    ``c_rank, c_row`` (this rank's expert-sorted slots), and the grouped layout ``tile_group, seg_start,
    seg_len`` of this rank's local experts; plus ``rows_all`` (padded rows of every rank)."""
    world, E = cnt_all.shape
    send_off = _excl_cumsum(cnt_all, 1)                                    # [world, E]
    seg_real = cnt_all.sum(0)                                              # [E]
    seg_len = (seg_real + ALIGN - 1) // ALIGN * ALIGN                      # [E]
    seg_start = _excl_cumsum(seg_len.reshape(world, El), 1).reshape(E)    # within each owner's layout
    rows_all = seg_len.reshape(world, El).sum(1)                           # [world]
    src_prefix = _excl_cumsum(cnt_all, 0)                                  # [world, E]: rows of lower sources
    # dispatch: owner `me`, experts e = me*El + j, pairs (j, src) expert-major
    lo = me * El
    cnt = cnt_all[:, lo:lo + El].T.reshape(-1)                             # [El*world]
    pos = (seg_start[lo:lo + El][:, None] + src_prefix[:, lo:lo + El].T).reshape(-1)
    soff = send_off[:, lo:lo + El].T.reshape(-1)
    srank = np.tile(np.arange(world), El)
    total = int(cnt.sum())
    within = np.arange(total) - np.repeat(_excl_cumsum(cnt), cnt)
    R = int(rows_all[me])
    d_rank = np.full(R, -1, dtype=np.int32)
    d_row = np.zeros(R, dtype=np.int32)
    dest = np.repeat(pos, cnt) + within
    d_rank[dest] = np.repeat(srank, cnt)
    d_row[dest] = np.repeat(soff, cnt) + within
    # combine: my slots sorted by expert
    mine = cnt_all[me]
    n = int(mine.sum())
    e_of = np.repeat(np.arange(E), mine)
    w_in = np.arange(n) - np.repeat(send_off[me], mine)
    c_rank = (e_of // El).astype(np.int32)
    c_row = (seg_start[e_of] + src_prefix[me, e_of] + w_in).astype(np.int32)
    tile_group = np.repeat(np.arange(El), seg_len[lo:lo + El] // ALIGN).astype(np.int32)
    return {"d_rank": d_rank, "d_row": d_row.astype(np.int32), "c_rank": c_rank, "c_row": c_row,
            "tile_group": tile_group, "seg_start": seg_start[lo:lo + El].astype(np.int32),
            "seg_len": seg_len[lo:lo + El].astype(np.int32), "rows_all": rows_all}


_RINGS: Dict[Any, ExchangeRing] = {}
_RETIRED: list = []  # rings replaced by larger ones, kept until teardown (pending backward passes use them)
_ENABLED = os.environ.get("RLB_EP_P2P", "1") != "0"


def set_enabled(flag: bool) -> None:
    global _ENABLED
    _ENABLED = bool(flag)


def usable(layer, xf: torch.Tensor) -> bool:
    g = layer.expert_group
    return (_ENABLED and available() and xf.is_cuda and xf.dtype == torch.bfloat16 and dist.is_initialized()
            and dist.get_backend(g) == "nccl" and layer._grouped_ready(xf))


def _ring_for(group, rows_needed: int, C: int, device) -> ExchangeRing:
    """The group's ring, replaced by a larger one when this call needs more rows (routing can concentrate
    on a few ranks).  Every rank computes ``rows_needed`` from the same all-gathered counts, so creating a
    ring -- a collective -- happens on every rank at the same call."""
    key = group if group is not None else "world"
    r = _RINGS.get(key)
    if r is None or r.C != C or rows_needed > r.slot_rows:
        if r is not None:
            _RETIRED.append(r)
        r = ExchangeRing(group, max(2 * rows_needed, 4096), C, device)
        _RINGS[key] = r
    return r


def close_all() -> None:
    for r in list(_RINGS.values()) + _RETIRED:
        r.close()
    _RINGS.clear()
    _RETIRED.clear()


def expert_parallel_moe_p2p(layer, xf: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor):
    """MoE layer over an expert-parallel group with peer-memory dispatch / combine (None: the exchange
    buffers could not be created on this node; the caller runs the NCCL path)."""
    from rl_project_b200.ops.grouped_gemm import GroupedLayout
    from rl_project_b200.ops.moe_dispatch import RowMaps, combine, dispatch

    group = layer.expert_group
    world, me = dist.get_world_size(group), dist.get_rank(group)
    E, k = layer.n_experts, indices.shape[1]
    El = E // world
    C = xf.shape[1]
    dev = xf.device
    flat = indices.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel(), device=dev)
    counts = torch.bincount(flat, minlength=E).to(torch.int32)
    cnt_all = torch.empty(world, E, dtype=torch.int32, device=dev)
    dist.all_gather_into_tensor(cnt_all, counts, group=group)
    cnt_np = cnt_all.cpu().numpy().astype(np.int64)  # the layer's one host synchronisation
    m = build_maps(cnt_np, me, El)
    need = int(max(cnt_np.sum(1).max(), m["rows_all"].max()))
    try:
        ring = _ring_for(group, need, C, dev)
    except Exception as e:  # no peer mapping on this node: fails alike on every rank, before its collectives
        import warnings

        warnings.warn(f"peer-memory expert exchange unavailable ({e}); using NCCL all-to-all")
        set_enabled(False)
        return None
    host = np.concatenate([m["d_rank"], m["d_row"], m["c_rank"], m["c_row"], m["tile_group"], m["seg_start"],
                           m["seg_len"]]).astype(np.int32)
    tab = torch.from_numpy(host).pin_memory().to(dev, non_blocking=True)
    sizes = [m["d_rank"].size, m["d_row"].size, m["c_rank"].size, m["c_row"].size, m["tile_group"].size,
             m["seg_start"].size, m["seg_len"].size]
    d_rank, d_row, c_rank, c_row, tile_group, seg_start, seg_len = torch.split(tab, sizes)
    maps = RowMaps(order.numel(), k, inv, order, torch.div(order, k, rounding_mode="floor"))
    xs = dispatch(xf, maps)  # my slots, expert-sorted (gather; the backward sums each token's k rows)
    xp = _Exchange.apply(xs, ring, d_rank, d_row, c_rank, c_row)
    R = int(m["rows_all"][me])
    layout = GroupedLayout(R, None, tile_group, seg_start, seg_len)
    first = layer.local_experts[0]
    if R:
        y = layer._experts_grouped(xp, layout, first, El)
    else:
        y = xp.new_zeros(0, C) + 0 * xp.sum()  # keeps the graph (and the exchange sequence) intact
    ys = _Exchange.apply(y, ring, c_rank, c_row, d_rank, d_row)
    return combine(ys, weights, maps)
