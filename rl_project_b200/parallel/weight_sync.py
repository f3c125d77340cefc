"""Weight broadcast from one rank to its group through NVSwitch multicast (comm path 5).

The reference synchronises rollout workers by shipping a full ``state_dict``
through Ray's object store (``src/forgeline/orchestration/ray_backend.py:408-417``)
and starts data-parallel ranks with one NCCL broadcast per parameter.  Here the
tensors are packed into chunks; for each chunk the source rank runs one kernel
that stores every 16-byte vector once to the NVLink multicast address of a
symmetric buffer (``multimem.st``), so the switch writes it into every rank's
copy and the source's NVLink egress is one copy whatever the group size.  A
device barrier (torch symmetric memory) then releases the ranks to unpack, and
a second one guards the buffer's reuse by the next chunk.

Without a multicast mapping -- gloo, one rank, no NVSwitch multicast on the
node, ``NCCL_NVLS_ENABLE=0`` in the environment (the switch this code honours
too, so failure tests run with no multicast binding), or fewer than
``min_world_multicast`` ranks, where multicast saves nothing -- every chunk is
one NCCL broadcast of the packed buffer instead of one broadcast per tensor.
"""

from __future__ import annotations

import os
from typing import Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from rl_project_b200.ops._ext import native
from rl_project_b200.observability.tracing import nvtx_annotate


def _byte_view(t: torch.Tensor) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError("broadcast tensors must be contiguous")
    return t.reshape(-1).view(torch.uint8)


class ParameterBroadcaster:
    def __init__(self, group=None, device: Optional[torch.device] = None, chunk_bytes: int = 256 << 20,
                 multicast: str = "auto", min_world_multicast: int = 4, barrier_timeout_ms: int = 120_000):
        if multicast not in ("auto", "on", "off"):
            raise ValueError("multicast must be auto|on|off")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.chunk = int(chunk_bytes) // 16 * 16
        self.device = device
        self.timeout_ms = int(barrier_timeout_ms)
        self.mode = "nccl" if dist.get_backend(group) == "nccl" else "host"
        self.h = None
        want = multicast == "on" or (multicast == "auto" and self.world >= min_world_multicast)
        if os.environ.get("NCCL_NVLS_ENABLE") == "0":
            want = False
        if want and self.mode == "nccl" and self.world > 1:
            import torch.distributed._symmetric_memory as symm

            g = group if group is not None else dist.group.WORLD
            buf = symm.empty(self.chunk, dtype=torch.uint8, device=device)
            h = symm.rendezvous(buf, g)
            mc = int(getattr(h, "multicast_ptr", 0) or 0)
            if mc:
                self.buf, self.h, self.mc, self.mode = buf, h, mc, "nvls"
            elif multicast == "on":
                raise RuntimeError("NVLink multicast requested but the node offers no multicast mapping")
        self.stage = torch.empty(self.chunk, dtype=torch.uint8, device=device) if self.mode != "host" else None

    def _pieces(self, tensors: Sequence[torch.Tensor]):
        """Yield lists of (byte view, offset in view, length) filling one chunk each."""
        cur: List[Tuple[torch.Tensor, int, int]] = []
        room = self.chunk
        for t in tensors:
            b = _byte_view(t)
            off = 0
            while off < b.numel():
                n = min(room, b.numel() - off)
                cur.append((b, off, n))
                off += n
                room -= n
                if room == 0:
                    yield cur
                    cur, room = [], self.chunk
        if cur:
            yield cur

    @torch.no_grad()
    @nvtx_annotate("rlb/param_broadcast")
    def broadcast_(self, tensors: Iterable[torch.Tensor], src: int = 0) -> None:
        tensors = [t for t in tensors]
        if self.world == 1 or not tensors:
            return
        if self.mode == "host":
            for t in tensors:
                dist.broadcast(t, src=src, group=self.group)
            return
        src_global = dist.get_global_rank(self.group, src) if self.group is not None else src
        for pieces in self._pieces(tensors):
            total = sum(n for _, _, n in pieces)
            padded = (total + 15) // 16 * 16
            if self.rank == src:
                pos = 0
                for b, off, n in pieces:
                    self.stage[pos:pos + n].copy_(b[off:off + n])
                    pos += n
            if self.mode == "nvls":
                if self.rank == src:
                    native().multimem_bcast(self.stage, self.mc, padded)
                self.h.barrier(0, self.timeout_ms)  # every copy of the chunk has landed
                data = self.buf
            else:
                dist.broadcast(self.stage[:padded], src=src_global, group=self.group)
                data = self.stage
            if self.rank != src:
                pos = 0
                for b, off, n in pieces:
                    b[off:off + n].copy_(data[pos:pos + n])
                    pos += n
            if self.mode == "nvls":
                self.h.barrier(0, self.timeout_ms)  # every rank unpacked before the buffer is reused


def broadcast_parameters(tensors: Iterable[torch.Tensor], group=None, src: int = 0, **kw) -> str:
    """Broadcast ``tensors`` in place from ``src``; returns the transport used (nvls / nccl / host)."""
    tensors = list(tensors)
    if not tensors:
        return "none"
    dev = tensors[0].device if tensors[0].is_cuda else None
    b = ParameterBroadcaster(group, device=dev, **kw)
    b.broadcast_(tensors, src=src)
    mode = b.mode
    if b.h is not None:
        torch.cuda.synchronize(dev)
    del b
    return mode
