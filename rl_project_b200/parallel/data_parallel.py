"""Data-parallel gradient synchronisation.

The reference broadcasts every parameter once and all-reduces every gradient
separately (``src/forgeline/training/common/trainer.py:122-139``).  Here
gradients are packed into flat buckets (``bucket_mb``, default 256 MB) so a
step issues a handful of large NCCL all-reduces instead of one per tensor;
averaging is folded into the pack (pre-divide by world size).
"""

from __future__ import annotations

from typing import List, Sequence

import torch
import torch.distributed as dist


def broadcast_parameters(params: Sequence[torch.nn.Parameter], strategy=None, src: int = 0) -> None:
    """Start every rank from ``src``'s weights: packed chunks through NVSwitch multicast or one NCCL broadcast
    per chunk (rl_project_b200/parallel/weight_sync.py)."""
    from rl_project_b200.parallel.weight_sync import broadcast_parameters as _bcast

    _bcast([p.data for p in params], src=src)


def _buckets(params: List[torch.nn.Parameter], cap_bytes: int, get) -> List[List[torch.nn.Parameter]]:
    out, cur, size, key = [], [], 0, None
    for p in params:
        t = get(p)
        k = (t.dtype, t.device)
        nb = t.numel() * t.element_size()
        if cur and (size + nb > cap_bytes or k != key):
            out.append(cur)
            cur, size = [], 0
        cur.append(p)
        size += nb
        key = k
    if cur:
        out.append(cur)
    return out


def all_reduce_gradients(params: Sequence[torch.nn.Parameter], strategy=None, bucket_mb: int = 256,
                         group=None) -> None:
    world = dist.get_world_size(group)
    ps = list(params)
    for p in ps:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
    for bucket in _buckets(ps, bucket_mb << 20, lambda p: p.grad):
        grads = [p.grad for p in bucket]
        flat = torch.cat([g.reshape(-1) for g in grads]) if len(grads) > 1 else grads[0].reshape(-1)
        flat.div_(world)
        dist.all_reduce(flat, group=group)
        if len(grads) > 1:
            off = 0
            for g in grads:
                n = g.numel()
                g.copy_(flat[off:off + n].view_as(g))
                off += n
