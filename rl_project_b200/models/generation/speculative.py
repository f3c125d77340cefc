"""Speculative decoding (Leviathan et al., 2023, "Fast Inference from Transformers
via Speculative Decoding"): a cheap proposer drafts ``k`` tokens, the target
scores all of them in one forward pass, each draft token is kept with
probability ``min(1, p_target / p_draft)``, the first rejection is resampled
from ``normalize(max(0, p_target - p_draft))``, and a fully accepted draft
earns one bonus token from the target.  Two proposers, as in
``src/forgeline/models/generation/speculative.py``: a separate draft model, or
the model's own multi-token-prediction heads (self-speculation).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn.functional as F


def _probs(logits: torch.Tensor, temperature: float, top_k: Optional[int]) -> torch.Tensor:
    x = logits.float() / temperature
    if top_k is not None:
        kth = torch.topk(x, min(top_k, x.shape[-1])).values[:, -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    return F.softmax(x, dim=-1)


def _accept_or_resample(idx: torch.Tensor, tok: torch.Tensor, p_t: torch.Tensor, p_d: torch.Tensor):
    """Returns (new idx, accepted?)."""
    ratio = (p_t.gather(1, tok) / (p_d.gather(1, tok) + 1e-10)).clamp(max=1.0)
    if torch.rand(1, device=idx.device) < ratio:
        return torch.cat([idx, tok], 1), True
    resid = (p_t - p_d).clamp(min=0)
    resid = resid / (resid.sum(-1, keepdim=True) + 1e-10)
    return torch.cat([idx, torch.multinomial(resid, 1)], 1), False


class SpeculativeGenerator:
    def __init__(self, target_model, draft_model, k: int = 5):
        self.target, self.draft, self.k = target_model, draft_model, k
        self.stats = {"proposed": 0, "accepted": 0}

    @torch.no_grad()
    def generate(self, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = 50):
        temperature = max(temperature, 1e-8)
        done = 0
        tb, db = self.target.spec.block_size, self.draft.spec.block_size
        while done < max_new_tokens:
            toks: List[torch.Tensor] = []
            qs: List[torch.Tensor] = []
            cur = idx
            for _ in range(self.k):
                logits, _ = self.draft(cur[:, -db:])
                q = _probs(logits[:, -1], temperature, top_k)
                t = torch.multinomial(q, 1)
                toks.append(t)
                qs.append(q)
                cur = torch.cat([cur, t], 1)
            seq = torch.cat([idx] + toks, 1)[:, -tb:]
            tlog = self.target.full_logits(seq)
            shift = seq.shape[1] - (idx.shape[1] + self.k)
            base = idx.shape[1] - 1 + shift
            all_ok = True
            for i in range(self.k):
                pos = base + i
                if pos < 0 or pos >= tlog.shape[1]:
                    all_ok = False
                    break
                self.stats["proposed"] += 1
                idx, ok = _accept_or_resample(idx, toks[i], _probs(tlog[:, pos], temperature, top_k), qs[i])
                done += 1
                if not ok:
                    all_ok = False
                    break
                self.stats["accepted"] += 1
                if done >= max_new_tokens:
                    break
            if all_ok and done < max_new_tokens and 0 <= base + self.k < tlog.shape[1]:
                idx = torch.cat([idx, torch.multinomial(_probs(tlog[:, base + self.k], temperature, top_k), 1)], 1)
                done += 1
            if idx.shape[1] >= tb:
                break
        return idx

    @property
    def acceptance_rate(self) -> float:
        return self.stats["accepted"] / max(self.stats["proposed"], 1)


class MTPSpeculativeGenerator:
    """Self-speculation: the main head samples token 1, each MTP depth drafts the next."""

    def __init__(self, model):
        if model.mtp_modules is None or len(model.mtp_modules) == 0:
            raise ValueError("MTPSpeculativeGenerator requires a model with n_predict_tokens > 1")
        self.model = model
        self.n_drafts = len(model.mtp_modules)

    @torch.no_grad()
    def generate(self, idx: torch.Tensor, max_new_tokens: int = 200, temperature: float = 1.0,
                 top_k: Optional[int] = 50):
        m = self.model.eval()
        temperature = max(temperature, 1e-8)
        block = m.spec.block_size
        done = 0
        while done < max_new_tokens:
            logits, _ = m(idx[:, -block:])
            h_last = m._last_hidden[:, -1:]
            p1 = _probs(logits[:, -1], temperature, top_k)
            first = torch.multinomial(p1, 1)
            drafts, dprobs = [], []
            emb = m.transformer.wte(first)
            for mod in m.mtp_modules:
                hm = mod(h_last, emb)
                q = _probs(m.logits(hm[:, -1]), temperature, top_k)
                t = torch.multinomial(q, 1)
                drafts.append(t)
                dprobs.append(q)
                emb = m.transformer.wte(t)
            idx = torch.cat([idx, first], 1)
            done += 1
            if done >= max_new_tokens:
                break
            if drafts:
                seq = torch.cat([idx] + drafts, 1)[:, -block:]
                vlog = m.full_logits(seq)
                shift = seq.shape[1] - (idx.shape[1] + len(drafts))
                for i, (t, q) in enumerate(zip(drafts, dprobs)):
                    if done >= max_new_tokens:
                        break
                    pos = idx.shape[1] - 1 + shift
                    if pos < 0 or pos >= vlog.shape[1]:
                        break
                    idx, ok = _accept_or_resample(idx, t, _probs(vlog[:, pos], temperature, top_k), q)
                    done += 1
                    if not ok:
                        break
            if idx.shape[1] >= block:
                break
        return idx
