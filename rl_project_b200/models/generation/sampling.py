"""Sampling filters and autoregressive generation for the model-level ``generate`` path (the serving and
rollout engines sample with the fused kernel in csrc/sampler.cu; these are the same filters in PyTorch).

Filter order (semantics of ``src/forgeline/models/generation/sampling.py``): repetition penalty,
temperature, top-k, min-p, top-p; temperature 0 means greedy.  ``apply_sampling_filters`` runs the stages
of ``_STAGES`` whose parameters are active, each on the output of the one before.

``generate_tokens`` writes into one preallocated ``[B, T + max_new]`` token buffer (no per-step
concatenation), keeps a per-row ``[B, V]`` seen-token mask for the repetition penalty (every row is
penalised by its own history -- the reference applies the penalty to single-row batches only; for one row
the two agree), and tests the batch-wide stop condition on the device, reading it back every
``sync_every`` steps.  Because the step at which every row had stopped is recorded on the device, the
returned tokens end exactly where a per-step check would have stopped.
"""

from __future__ import annotations

from typing import Callable, Iterable, List, Optional, Sequence, Tuple

import torch

_NEG = float("-inf")


def _penalise(x: torch.Tensor, seen: torch.Tensor, penalty: float) -> torch.Tensor:
    """Shrink the logits of already-seen tokens toward zero by ``penalty`` (divide positives, multiply
    negatives)."""
    scaled = torch.where(x > 0, x / penalty, x * penalty)
    return torch.where(seen, scaled, x)


def _top_k(x: torch.Tensor, k: int) -> torch.Tensor:
    kth = torch.topk(x, min(k, x.shape[-1]), dim=-1).values[..., -1:]
    return x.masked_fill(x < kth, _NEG)


def _min_p(x: torch.Tensor, p_min: float) -> torch.Tensor:
    p = x.softmax(-1)
    return x.masked_fill(p < p_min * p.amax(-1, keepdim=True), _NEG)


def _top_p(x: torch.Tensor, p_top: float) -> torch.Tensor:
    """Nucleus: keep, in descending order, every token whose preceding probability mass is below ``p_top``."""
    vals, order = x.sort(-1, descending=True)
    probs = vals.softmax(-1)
    vals = vals.masked_fill(probs.cumsum(-1) - probs >= p_top, _NEG)
    return torch.empty_like(x).scatter_(-1, order, vals)


# (is the stage active for these settings, stage)
_STAGES: List[Tuple[Callable[[dict], bool], Callable[[torch.Tensor, dict], torch.Tensor]]] = [
    (lambda s: s["penalty"] != 1.0 and s["seen"] is not None, lambda x, s: _penalise(x, s["seen"], s["penalty"])),
    (lambda s: s["temperature"] > 0, lambda x, s: x / s["temperature"]),
    (lambda s: bool(s["top_k"]) and s["top_k"] > 0, lambda x, s: _top_k(x, s["top_k"])),
    (lambda s: bool(s["min_p"]) and s["min_p"] > 0, lambda x, s: _min_p(x, s["min_p"])),
    (lambda s: s["top_p"] is not None and 0 < s["top_p"] < 1.0, lambda x, s: _top_p(x, s["top_p"])),
]


def _seen_mask(rows: int, vocab: int, device, tokens: Optional[torch.Tensor]) -> torch.Tensor:
    seen = torch.zeros(rows, vocab, dtype=torch.bool, device=device)
    if tokens is not None and tokens.numel():
        seen.scatter_(1, tokens.to(device).long().view(rows if tokens.dim() > 1 else 1, -1).expand(rows, -1), True)
    return seen


def apply_sampling_filters(logits: torch.Tensor, temperature: float = 1.0, top_k: Optional[int] = None,
                           top_p: Optional[float] = None, min_p: Optional[float] = None,
                           repetition_penalty: float = 1.0, past_tokens: Optional[Sequence[int]] = None,
                           seen: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Filtered ``[B, V]`` logits.  The penalty applies to ``seen`` (a ``[B, V]`` bool mask, one history per
    row) or, given ``past_tokens``, to those ids in every row."""
    if seen is None and past_tokens:
        seen = _seen_mask(logits.shape[0], logits.shape[-1], logits.device,
                          torch.as_tensor(list(past_tokens), dtype=torch.long))
    settings = {"penalty": repetition_penalty, "seen": seen, "temperature": temperature, "top_k": top_k,
                "min_p": min_p, "top_p": top_p}
    x = logits
    for active, stage in _STAGES:
        if active(settings):
            x = stage(x, settings)
    return x.clone() if x is logits else x


def sample_from_logits(logits: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """``[B, 1]`` token ids: argmax at temperature 0, else one multinomial draw from the softmax."""
    if temperature <= 0:
        return logits.argmax(-1, keepdim=True)
    return torch.multinomial(logits.float().softmax(-1), 1)


@torch.no_grad()
def generate_tokens(model, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
                    top_k: Optional[int] = None, top_p: Optional[float] = None, min_p: Optional[float] = None,
                    repetition_penalty: float = 1.0, use_cache: bool = True, stop_token_ids: Iterable[int] = (),
                    return_logprobs: bool = False, sync_every: Optional[int] = None):
    """Sample up to ``max_new_tokens`` continuations of ``idx [B, T]``; returns ``[B, T + R]`` (and the
    sampled tokens' log-probs ``[B, R]`` under the filtered distribution when ``return_logprobs``).
    With ``use_cache`` the model's ``prefill`` / ``step`` KV-cache path runs (one position per step) until
    the context reaches ``block_size``; otherwise the last ``block_size`` tokens are re-run each step."""
    dev = idx.device
    B, T = idx.shape
    block = model.spec.block_size
    stop = torch.as_tensor(sorted({int(t) for t in stop_token_ids}), dtype=torch.long, device=dev)
    every = sync_every or (8 if dev.type == "cuda" else 1)
    tokens = torch.empty(B, T + max_new_tokens, dtype=idx.dtype, device=dev)
    tokens[:, :T] = idx
    lps = torch.zeros(B, max_new_tokens, device=dev) if return_logprobs else None
    seen = None  # [B, V] seen-token mask, built on the first step (V = the logits' width)
    done = torch.zeros(B, dtype=torch.bool, device=dev)
    all_done_at = torch.full((), max_new_tokens, dtype=torch.long, device=dev)  # steps kept

    cached = use_cache and T < block
    if cached:
        logits, cache = model.prefill(idx)
    n = 0
    while n < max_new_tokens:
        if not cached:
            lo = max(0, T + n - block)
            logits = model(tokens[:, lo:T + n])[0][:, -1]
        if repetition_penalty != 1.0 and seen is None:
            seen = _seen_mask(B, logits.shape[-1], dev, idx)
        filt = apply_sampling_filters(logits.float(), temperature, top_k, top_p, min_p, repetition_penalty, seen=seen)
        nxt = sample_from_logits(filt, temperature)
        tokens[:, T + n] = nxt[:, 0]
        if lps is not None:
            lps[:, n] = filt.log_softmax(-1).gather(1, nxt)[:, 0]
        if seen is not None:
            seen.scatter_(1, nxt, True)
        n += 1
        if stop.numel():
            done |= torch.isin(nxt[:, 0], stop)
            all_done_at = torch.where(done.all() & (all_done_at == max_new_tokens), torch.full_like(all_done_at, n),
                                      all_done_at)
            if n % every == 0 and int(all_done_at) < max_new_tokens:
                break
        if cached:
            pos = T + n - 1  # position of the token just sampled
            if pos >= block:
                break
            logits, cache = model.step(nxt, cache, pos)
    kept = min(n, int(all_done_at)) if stop.numel() else n
    out = tokens[:, :T + kept]
    if lps is not None:
        return out, lps[:, :kept]
    return out
