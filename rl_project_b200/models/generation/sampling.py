"""Sampling filters and autoregressive generation
(``src/forgeline/models/generation/sampling.py:16-132`` semantics: repetition
penalty, temperature, top-k, min-p, top-p, in that order; greedy at
temperature 0; batch-wide early stop once every row produced a stop token).
The stop test runs on the device (one boolean read per step instead of a
Python loop over the batch)."""

from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F


def apply_sampling_filters(logits: torch.Tensor, temperature: float = 1.0, top_k: Optional[int] = None,
                           top_p: Optional[float] = None, min_p: Optional[float] = None,
                           repetition_penalty: float = 1.0,
                           past_tokens: Optional[Sequence[int]] = None) -> torch.Tensor:
    x = logits.clone()
    if repetition_penalty != 1.0 and past_tokens:
        ids = torch.as_tensor(list(past_tokens), device=x.device).unique()
        sel = x[:, ids]
        x[:, ids] = torch.where(sel > 0, sel / repetition_penalty, sel * repetition_penalty)
    if temperature > 0:
        x = x / temperature
    if top_k is not None and top_k > 0:
        kth = torch.topk(x, min(top_k, x.shape[-1])).values[:, -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    if min_p is not None and min_p > 0:
        p = F.softmax(x, dim=-1)
        x = x.masked_fill(p < min_p * p.amax(-1, keepdim=True), float("-inf"))
    if top_p is not None and 0 < top_p < 1.0:
        sx, si = torch.sort(x, descending=True)
        sp = F.softmax(sx, dim=-1)
        drop = (sp.cumsum(-1) - sp) >= top_p
        sx = sx.masked_fill(drop, float("-inf"))
        x = sx.scatter(1, si, sx)
    return x


def sample_from_logits(logits: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    if temperature <= 0:
        return logits.argmax(-1, keepdim=True)
    return torch.multinomial(F.softmax(logits.float(), dim=-1), 1)


@torch.no_grad()
def generate_tokens(model, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
                    top_k: Optional[int] = None, top_p: Optional[float] = None, min_p: Optional[float] = None,
                    repetition_penalty: float = 1.0, use_cache: bool = True, stop_token_ids: Iterable[int] = (),
                    return_logprobs: bool = False):
    stop = torch.as_tensor(sorted({int(t) for t in stop_token_ids}), device=idx.device, dtype=torch.long)
    B = idx.shape[0]
    past: Optional[List[int]] = idx[0].tolist() if (repetition_penalty != 1.0 and B == 1) else None
    out: List[torch.Tensor] = []
    lps: List[torch.Tensor] = []
    done = torch.zeros(B, dtype=torch.bool, device=idx.device)
    block = model.spec.block_size

    def pick(logits: torch.Tensor) -> torch.Tensor:
        f = apply_sampling_filters(logits.float(), temperature, top_k, top_p, min_p, repetition_penalty, past)
        nxt = sample_from_logits(f, temperature)
        if return_logprobs:
            lps.append(F.log_softmax(f, -1).gather(1, nxt).squeeze(1))
        return nxt

    def finished(nxt: torch.Tensor) -> bool:
        nonlocal done
        if stop.numel():
            done = done | torch.isin(nxt.squeeze(1), stop)
            return bool(done.all())
        return False

    if use_cache and idx.shape[1] < block:
        logits, cache = model.prefill(idx)
        pos = idx.shape[1]
        for _ in range(max_new_tokens):
            nxt = pick(logits)
            out.append(nxt)
            if past is not None:
                past.append(int(nxt.item()))
            if finished(nxt) or pos >= block:
                break
            logits, cache = model.step(nxt, cache, pos)
            pos += 1
    else:
        seq = idx
        for _ in range(max_new_tokens):
            ctx = seq if seq.shape[1] <= block else seq[:, -block:]
            logits, _ = model(ctx)
            nxt = pick(logits[:, -1, :])
            out.append(nxt)
            seq = torch.cat([seq, nxt], 1)
            if past is not None:
                past.append(int(nxt.item()))
            if finished(nxt):
                break
    full = torch.cat([idx] + out, 1) if out else idx
    if return_logprobs:
        return full, (torch.stack(lps, 1) if lps else torch.zeros(B, 0, device=idx.device))
    return full
