"""Reduce-scatter of sharded-data-parallel gradients over NVLink peer memory,
fused with the fp32 cast, the 1/world average, accumulation into the shard
gradient and the squared-norm partial (kernel: csrc/comm_fused.cu).

The reference reduces FSDP gradients through torch FSDP's NCCL reduce-scatter
(``src/forgeline/training/common/trainer.py:108-170`` wraps the model in
``FullyShardedDataParallel``), then casts, averages and clips in separate
passes.  Here one kernel per unit reads the owned slice of every rank's bf16
gradient straight out of the peers' memory -- or has the NVSwitch add the
copies (``multimem.ld_reduce`` through the buffer's multicast address) -- and
writes the fp32 shard gradient and its squared norm.

Buffers.  A peer-visible allocation (plain cudaMalloc memory mapped into the
other ranks with CUDA IPC, or torch symmetric memory when the NVLink multicast
address is wanted) holds ``NSLOTS`` gradient slots of ``slot_elems`` bf16
each, and a peer-visible int32 flag array ``[NSLOTS, world]``.
Units take slots round-robin by a sequence number ``q`` that every rank
advances identically (collectives are issued in the same order on all ranks,
as NCCL requires too); the slot's epoch is ``q // NSLOTS + 1``.

Protocol for unit ``q`` on rank ``r`` (slot ``s = q % NSLOTS``):

1. compute stream: wait for this rank's reduce ``q - LAG`` (an event), then
   pack the gradients into slot ``s``;
2. communication stream (after the compute stream): ``signal`` stores the
   epoch into flag ``[s, r]`` of every rank (release, system scope), then the
   reduce waits (bounded) until flag ``[s, p] >= epoch`` for every ``p`` and
   reads slice ``r`` of slot ``s`` from every rank.

Why a slot is never overwritten while a peer still reads it: rank A refills
slot ``s`` for ``q`` only after A's reduce ``q - 3`` finished, which needed
peer B's signal ``q - 3``; B issues that signal on its communication stream
after its reduce ``q - 4`` -- the last reader of slot ``s`` before ``q`` -- has
finished.  With ``NSLOTS = 4`` and ``LAG = 3`` the compute stream never waits
on the reduce that was just issued, only on one three units back.
Conversely B cannot refill slot ``s`` (for ``q + 4``) before A's reduce ``q``
finished, since that needs A's signal ``q + 1``, issued after A's reduce ``q``.

Every wait in the kernel is bounded by ``timeout_s``; a timeout leaves the
output untouched and sets a status word that ``check`` raises as
``DistributedTimeoutError`` (and that turns the gradient norm into NaN, so
the optimizer skips the step).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.distributed as dist

from rl_project_b200.core.errors import DistributedConfigError, DistributedTimeoutError
from rl_project_b200.ops._ext import native
from rl_project_b200.observability.tracing import nvtx_annotate

NSLOTS = 4
LAG = 3
ALIGN = 8  # elements: a shard is a whole number of 16-byte vectors


def available(group=None) -> bool:
    """True when the group's ranks are NCCL ranks on CUDA devices of this node (peer-mappable memory)."""
    if not (dist.is_available() and dist.is_initialized() and torch.cuda.is_available()):
        return False
    if dist.get_backend(group) != "nccl":
        return False
    import os

    world = dist.get_world_size(group)
    return int(os.environ.get("LOCAL_WORLD_SIZE", world)) >= world  # torchrun sets it; one node assumed otherwise


class _IpcBuffers:
    """Slots and flags in plain cudaMalloc allocations of whole 2 MiB pages, mapped into every peer with CUDA
    IPC (no multicast object is bound to them, so only peer loads are possible).  A handle names the whole
    allocation; each rank sends its buffer's offset in it along with the handle."""

    def __init__(self, group, nbytes_buf: int, nbytes_flags: int, device: torch.device):
        C = native()
        self.device = device
        dev = device.index if device.index is not None else torch.cuda.current_device()
        self.dev = dev
        self.buf_raw = C.peer_alloc(nbytes_buf, dev)
        self.flags_raw = C.peer_alloc(nbytes_flags, dev)
        mine = (C.peer_handle(self.buf_raw), C.peer_handle(self.flags_raw))
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        handles: list = [None] * world
        dist.all_gather_object(handles, mine, group=group)
        self.opened = []
        self.buffer_ptrs, self.flag_ptrs = [], []
        for p, ((hb, ob), (hf, of)) in enumerate(handles):
            if p == rank:
                self.buffer_ptrs.append(self.buf_raw.data_ptr())
                self.flag_ptrs.append(self.flags_raw.data_ptr())
            else:
                pb, pf = C.peer_open(hb, dev), C.peer_open(hf, dev)  # mapping bases; buffers sit at an offset
                self.opened += [pb, pf]
                self.buffer_ptrs.append(pb + ob)
                self.flag_ptrs.append(pf + of)
        for ptr in self.buffer_ptrs + self.flag_ptrs:
            if ptr % 16:
                raise DistributedConfigError(f"peer buffer at 0x{ptr:x} is not 16-byte aligned")
        self.multicast_ptr = 0
        self.group = group

    def close(self) -> None:
        C = native()
        torch.cuda.synchronize(self.device)
        for ptr in self.opened:
            C.peer_close(ptr, self.dev)
        self.opened = []
        dist.barrier(group=self.group)  # no peer maps this rank's buffers any more


class _SymmBuffers:
    """Slots and flags in torch symmetric memory (with an NVLink multicast mapping when the node has one)."""

    def __init__(self, group, nbytes_buf: int, nbytes_flags: int, device: torch.device):
        import torch.distributed._symmetric_memory as symm

        group = group if group is not None else dist.group.WORLD
        self.buf_raw = symm.empty(nbytes_buf, dtype=torch.uint8, device=device)
        self.buf_raw.zero_()
        self.h = symm.rendezvous(self.buf_raw, group)
        self.flags_raw = symm.empty(nbytes_flags, dtype=torch.uint8, device=device)
        self.flags_raw.zero_()
        self.hf = symm.rendezvous(self.flags_raw, group)
        self.buffer_ptrs = [int(x) for x in self.h.buffer_ptrs]
        self.flag_ptrs = [int(x) for x in self.hf.buffer_ptrs]
        self.multicast_ptr = int(getattr(self.h, "multicast_ptr", 0) or 0)
        self.group = group
        self.device = device

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


class FusedReduceScatter:
    """Ring of peer-visible bf16 gradient slots plus flags; one fused reduce per unit.

    ``multicast``: ``off`` (default) maps the peers' buffers with CUDA IPC and sums with peer loads; ``on``
    allocates torch symmetric memory and sums through its NVLink multicast address (``multimem.ld_reduce``);
    ``symm`` uses symmetric memory with peer loads."""

    def __init__(self, group, slot_elems: int, device: torch.device, multicast: str = "off",
                 timeout_s: float = 120.0, ctas: int = 32):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if slot_elems % (ALIGN * self.world):
            raise DistributedConfigError(f"slot size {slot_elems} is not a multiple of {ALIGN} x world")
        if multicast not in ("off", "on", "symm"):
            raise DistributedConfigError(f"multicast must be off|on|symm, got {multicast!r}")
        self.slot_elems = int(slot_elems)
        self.device = device
        nb, nf = NSLOTS * self.slot_elems * 2, NSLOTS * self.world * 4
        self.mem = _IpcBuffers(group, nb, nf, device) if multicast == "off" else _SymmBuffers(group, nb, nf, device)
        self.buf = self.mem.buf_raw.view(torch.bfloat16)
        self.flags = self.mem.flags_raw.view(torch.int32)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        bytes_per_slot = self.slot_elems * 2
        self.ptrs = torch.tensor([[self.mem.buffer_ptrs[p] + s * bytes_per_slot for p in range(self.world)]
                                  for s in range(NSLOTS)], dtype=torch.int64, device=device)
        self.flag_ptrs = torch.tensor(self.mem.flag_ptrs, dtype=torch.int64, device=device)
        mc = self.mem.multicast_ptr if multicast == "on" else 0
        if multicast == "on" and not mc:
            raise DistributedConfigError("NVLink multicast was requested but the buffer has no multicast mapping")
        self.mc = mc
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=device)
        self.limit_ns = int(timeout_s * 1e9)
        self.ctas = int(ctas)
        self.seq = 0
        self.events: Dict[int, torch.cuda.Event] = {}

    @property
    def uses_multicast(self) -> bool:
        return self.mc != 0

    def next_slot(self, numel: int) -> torch.Tensor:
        """The slot the next unit packs its gradients into (``numel`` elements), after the current stream
        waited for this rank's reduce ``LAG`` units back."""
        if numel > self.slot_elems:
            raise DistributedConfigError(f"unit of {numel} elements exceeds the slot size {self.slot_elems}")
        ev = self.events.pop(self.seq - LAG, None)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
        s = self.seq % NSLOTS
        return self.buf[s * self.slot_elems: s * self.slot_elems + numel]

    @nvtx_annotate("rlb/fused_reduce_scatter")
    def reduce(self, shard: int, out: torch.Tensor, accumulate: bool, norm: bool,
               stream: Optional[torch.cuda.Stream] = None, ctas: Optional[int] = None) -> None:
        """Signal the peers that this rank's slot is filled, then reduce slice ``rank`` of it into ``out``
        (fp32, ``shard`` elements): ``out (+)= sum_p slot_p / world``; squares added to ``sumsq`` if ``norm``."""
        if shard % ALIGN or shard * self.world > self.slot_elems or out.numel() != shard:
            raise DistributedConfigError(f"fused reduce of {shard} x {self.world} elements does not fit the slot "
                                         f"({self.slot_elems}) or the output ({out.numel()})")
        C = native()
        q = self.seq
        s = q % NSLOTS
        epoch = q // NSLOTS + 1
        stream = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(stream):
            C.signal_peers(self.flag_ptrs, self.rank, s, epoch)
            mc = self.mc + s * self.slot_elems * 2 if self.mc else 0
            C.fused_reduce_scatter(self.ptrs[s], mc, self.flags, self.rank, s, epoch, shard, 1.0 / self.world, out,
                                   accumulate, self.sumsq if norm else None, self.status, self.limit_ns,
                                   int(ctas or self.ctas))
            ev = torch.cuda.Event()
            ev.record(stream)
        self.events[q] = ev
        self.seq += 1

    def reset_norm(self) -> None:
        self.sumsq.zero_()

    def poll_status(self) -> None:
        """Queue a copy of the status word to pinned host memory (read by ``check`` after the next sync)."""
        self._status_host.copy_(self.status, non_blocking=True)

    def check(self) -> None:
        code = int(self._status_host.item())
        if code:
            raise DistributedTimeoutError(
                f"fused reduce-scatter: a peer's gradient flag did not arrive within the time limit "
                f"(status 0x{code:x}, slot {code >> 8})",
                hint="A rank stopped or fell behind; check the other ranks' logs.")

    def close(self) -> None:
        """Collective: unmap the peers' buffers on every rank before any rank frees its own."""
        self.events.clear()
        if self.mem is not None:
            self.mem.close()
            self.mem = None


class FusedAllGather:
    """All-gather of equal bf16 shards over peer memory (FSDP parameter gather).

    Each call copies this rank's shard into its slot of a CUDA-IPC ring, raises its flag for the slot on
    every rank, waits (bounded, one thread) for every peer's flag and pulls all shards into the full
    buffer with one kernel.  Calls are issued in the same order on every rank and on one stream, so a
    rank refills a slot only after its previous pull -- which needed every peer's newer signal, raised
    after that peer's own earlier pulls -- finished."""

    def __init__(self, group, max_shard: int, device: torch.device, timeout_s: float = 120.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_shard = (int(max_shard) + ALIGN - 1) // ALIGN * ALIGN
        self.device = device
        self.mem = _IpcBuffers(group, NSLOTS * self.max_shard * 2, NSLOTS * self.world * 4, device)
        self.buf = self.mem.buf_raw.view(torch.bfloat16).view(NSLOTS, self.max_shard)
        self.flags = self.mem.flags_raw.view(torch.int32)
        self.flags.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        slot_bytes = self.max_shard * 2
        self.bases = torch.tensor([[b + s * slot_bytes for b in self.mem.buffer_ptrs] for s in range(NSLOTS)],
                                  dtype=torch.int64, device=device)
        self.flag_ptrs = torch.tensor(self.mem.flag_ptrs, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.limit_ns = int(timeout_s * 1e9)
        self.seq = 0

    @nvtx_annotate("rlb/fused_all_gather")
    def gather(self, shard: torch.Tensor, full: torch.Tensor) -> None:
        """``full [world * S] = cat(every rank's shard [S])`` on the current stream."""
        C = native()
        S = shard.numel()
        if S > self.max_shard or S % ALIGN or full.numel() != S * self.world:
            raise DistributedConfigError(f"all-gather of {S} x {self.world} does not fit ({self.max_shard})")
        q = self.seq
        s, epoch = q % NSLOTS, q // NSLOTS + 1
        self.seq += 1
        self.buf[s, :S].copy_(shard.reshape(-1))
        C.signal_peers(self.flag_ptrs, self.rank, s, epoch)
        C.wait_peers(self.flags, self.world, s, epoch, self.limit_ns, self.status)
        C.allgather_pull(self.bases[s], S, full.reshape(-1))

    def check(self) -> None:
        if int(self.status.item()):
            raise DistributedTimeoutError("fused all-gather: a peer's flag did not arrive in time",
                                          hint="A rank stopped or fell behind; check the other ranks' logs.")

    def close(self) -> None:
        if self.mem is not None:
            self.mem.close()
            self.mem = None
