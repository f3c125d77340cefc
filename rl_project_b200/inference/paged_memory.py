"""Paged KV cache: block accounting (with shared prefixes) and the device pool.

The reference (``src/forgeline/inference/paged_memory.py:20-75``) only counts
blocks while every sequence keeps its own contiguous cache tensor.  Here the
blocks are real: ``PagedKVCache`` holds one ``[num_blocks, Hkv, 16, D]`` bf16
pool per layer for K and V, sequences address it through block tables, and
the decode kernel (csrc/paged_attention.cu) reads it directly, so sequences
of different lengths decode in one batch and nothing is concatenated or split.

``PagedBlockAllocator`` keeps the reference's interface (``blocks_needed``,
``can_allocate``, ``allocate``, ``append_token``, ``free``, ``stats``) and adds
reference counts: ``share_prefix`` lets a new sequence reuse the blocks of a
running one that has the same prompt (the G samples of one GRPO prompt are
prefilled once), and ``append_token`` copies a shared, partly filled last
block before the sequence writes into it (copy-on-write).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from rl_project_b200.core.errors import ServingError

KERNEL_BLOCK = 16  # tokens per block of the device kernels


class OutOfBlocksError(ServingError):
    hint = "Increase max_blocks / reduce max_batch, or wait for running sequences to finish."


class PagedBlockAllocator:
    def __init__(self, block_size: int = 16, max_blocks: int = 1024):
        if block_size < 1 or max_blocks < 1:
            raise ServingError("block_size and max_blocks must be >= 1")
        self.block_size = block_size
        self.max_blocks = max_blocks
        self.free_blocks: List[int] = list(range(max_blocks - 1, -1, -1))  # pop() hands out 0, 1, 2, ...
        self.tables: Dict[str, List[int]] = {}
        self.lengths: Dict[str, int] = {}
        self.refs: List[int] = [0] * max_blocks
        self.cow_copies = 0

    # ------------------------------------------------------------ accounting
    def blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    def can_allocate(self, seq_id: str, n_tokens: int) -> bool:
        have = len(self.tables.get(seq_id, []))
        return self.blocks_needed(n_tokens) - have <= len(self.free_blocks)

    def _take(self) -> int:
        b = self.free_blocks.pop()
        self.refs[b] = 1
        return b

    def _release(self, b: int) -> None:
        self.refs[b] -= 1
        if self.refs[b] == 0:
            self.free_blocks.append(b)

    def allocate(self, seq_id: str, n_tokens: int) -> List[int]:
        """Ensure ``seq_id`` owns enough blocks for ``n_tokens``; returns its block table."""
        table = self.tables.setdefault(seq_id, [])
        need = self.blocks_needed(n_tokens) - len(table)
        if need > len(self.free_blocks):
            raise OutOfBlocksError(f"sequence {seq_id} needs {need} more blocks, {len(self.free_blocks)} free")
        for _ in range(max(need, 0)):
            table.append(self._take())
        self.lengths[seq_id] = n_tokens
        return table

    def append_token(self, seq_id: str) -> Optional[Tuple[int, int]]:
        """Reserve the slot of one more token.

        Returns ``(src, dst)`` when the slot lies in a block shared with another
        sequence: the caller must copy block ``src`` to ``dst`` before writing.
        """
        n = self.lengths.get(seq_id, 0)
        table = self.tables.setdefault(seq_id, [])
        if n % self.block_size != 0 and table and self.refs[table[-1]] > 1:
            if not self.free_blocks:
                raise OutOfBlocksError(f"sequence {seq_id} needs a copy-on-write block, none free")
            src = table[-1]
            dst = self._take()
            self._release(src)
            table[-1] = dst
            self.lengths[seq_id] = n + 1
            self.cow_copies += 1
            return src, dst
        self.allocate(seq_id, n + 1)
        return None

    def share_prefix(self, parent_id: str, child_id: str, n_tokens: int) -> List[int]:
        """Make ``child_id`` start with the first ``n_tokens`` tokens of ``parent_id``.

        Any blocks the child held are released; the parent's blocks covering the
        prefix gain a reference instead of being copied.
        """
        parent = self.tables.get(parent_id)
        if parent is None or self.lengths.get(parent_id, 0) < n_tokens:
            raise ServingError(f"sequence {parent_id} does not hold a {n_tokens}-token prefix")
        self.free(child_id)
        shared = parent[: self.blocks_needed(n_tokens)]
        for b in shared:
            self.refs[b] += 1
        self.tables[child_id] = list(shared)
        self.lengths[child_id] = n_tokens
        return self.tables[child_id]

    def free(self, seq_id: str) -> None:
        for b in self.tables.pop(seq_id, []):
            self._release(b)
        self.lengths.pop(seq_id, None)

    @property
    def used_blocks(self) -> int:
        return self.max_blocks - len(self.free_blocks)

    @property
    def utilization(self) -> float:
        return self.used_blocks / self.max_blocks

    def stats(self) -> Dict[str, float]:
        return {"used_blocks": self.used_blocks, "free_blocks": len(self.free_blocks),
                "utilization": self.utilization, "sequences": len(self.tables),
                "shared_blocks": sum(1 for r in self.refs if r > 1), "cow_copies": self.cow_copies}


class PagedKVCache:
    """Device K/V pools ``[n_layer, num_blocks, Hkv, 16, D]`` addressed by block tables."""

    def __init__(self, n_layer: int, n_kv_head: int, head_dim: int, num_blocks: int,
                 device: torch.device, dtype: torch.dtype = torch.bfloat16, block_size: int = KERNEL_BLOCK):
        if block_size != KERNEL_BLOCK:
            raise ServingError(f"the paged KV cache uses {KERNEL_BLOCK}-token blocks (got {block_size})")
        shape = (n_layer, num_blocks, n_kv_head, block_size, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.block_size = block_size
        self.num_blocks = num_blocks

    def layer(self, i: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.k[i], self.v[i]

    @property
    def nbytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()

    def copy_block(self, src: int, dst: int) -> None:
        self.k[:, dst].copy_(self.k[:, src])
        self.v[:, dst].copy_(self.v[:, src])

    def write_prefix(self, layer: int, k: torch.Tensor, v: torch.Tensor, table: List[int]) -> None:
        """Store a prompt's keys/values ``[Hkv, T, D]`` (positions 0..T-1) into its blocks."""
        from rl_project_b200.ops.paged_attention import paged_write

        T = k.shape[1]
        pos = torch.arange(T)
        blocks = torch.as_tensor(table, dtype=torch.int32)[pos // self.block_size]
        offs = (pos % self.block_size).to(torch.int32)
        dev = self.k.device
        kl, vl = self.layer(layer)
        paged_write(k.transpose(0, 1), v.transpose(0, 1), kl, vl, blocks.to(dev, non_blocking=True),
                    offs.to(dev, non_blocking=True))
