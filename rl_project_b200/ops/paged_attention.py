"""Paged-KV decode attention and slot writes (csrc/paged_attention.cu).

KV pools are ``[num_blocks, Hkv, BLOCK, D]`` bf16 per layer (BLOCK = 16 tokens);
each sequence owns a row of ``block_tables [B, max_blocks]`` (int32) and a
context length ``ctx_lens [B]`` (int32, including the token being decoded).
On CUDA both ops run the native kernels (and raise if the extension is
missing); on CPU they run the plain-PyTorch reference below, which is also the
numerics oracle of the GPU tests.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_project_b200.ops._ext import native

BLOCK = 16


def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_tables: torch.Tensor,
                 ctx_lens: torch.Tensor, scale: float, softcap: float = 0.0, window: int = 0,
                 split_tokens: int = 0, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query token per sequence: ``q [B, Hq, D]`` -> ``[B, Hq, D]``.

    ``split_tokens > 0`` splits each context into chunks of that many tokens
    processed by separate CTAs and merged afterwards (long contexts, few
    sequences); 0 processes a whole context in one CTA per (kv head, sequence).
    """
    if q.is_cuda:
        return native().paged_decode(q.contiguous(), k_pool, v_pool, block_tables, ctx_lens, int(split_tokens),
                                     float(scale), float(softcap), int(window), status)
    return paged_decode_reference(q, k_pool, v_pool, block_tables, ctx_lens, scale, softcap, window)


def paged_write(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                slot_block: torch.Tensor, slot_off: torch.Tensor, status: Optional[torch.Tensor] = None) -> None:
    """Write row ``i`` of ``k_new/v_new [N, Hkv, D]`` into block ``slot_block[i]``, offset ``slot_off[i]``."""
    if k_new.is_cuda:
        native().paged_write(k_new.contiguous(), v_new.contiguous(), k_pool, v_pool, slot_block, slot_off, status)
        return
    blk, off = slot_block.long(), slot_off.long()
    k_pool[blk, :, off] = k_new.to(k_pool.dtype)
    v_pool[blk, :, off] = v_new.to(v_pool.dtype)


def paged_decode_reference(q, k_pool, v_pool, block_tables, ctx_lens, scale, softcap=0.0, window=0):
    B, Hq, D = q.shape
    Hkv = k_pool.shape[1]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(ctx_lens[b])
        if n <= 0:
            continue
        blocks = block_tables[b, : (n + BLOCK - 1) // BLOCK].long()
        k = k_pool[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :n].float().repeat_interleave(G, 0)
        v = v_pool[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :n].float().repeat_interleave(G, 0)
        s = torch.einsum("hd,htd->ht", q[b].float(), k) * scale
        if softcap > 0:
            s = torch.tanh(s / softcap) * softcap
        if window > 0 and n > window:
            s[:, : n - window] = float("-inf")
        out[b] = torch.einsum("ht,htd->hd", s.softmax(-1), v)
    return out.to(q.dtype)
