"""Fused temperature sampling (csrc/sampler.cu).

``sample_tokens(logits [B, V], temperature [B], seed)`` returns ``(tokens [B]
int64, logprobs [B] fp32)``: an exact draw from ``softmax(logits / T)`` by the
Gumbel-max identity with counter-hashed noise (``T = 0``: argmax, log-prob
under ``T = 1``).  One read of the logits; no probability tensor, no
multinomial.  CUDA runs the kernel; CPU runs the same identity with torch ops
(independent noise, same distribution).
"""

from __future__ import annotations

from typing import Tuple

import torch

from rl_project_b200.ops._ext import native


def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor, seed: int) -> Tuple[torch.Tensor, torch.Tensor]:
    if logits.is_cuda:
        x = logits if logits.stride(-1) == 1 else logits.contiguous()
        t = temperature.to(device=logits.device, dtype=torch.float32)
        tok, lp = native().sample(x, t, int(seed) & ((1 << 63) - 1))
        return tok, lp
    x = logits.float()
    t = temperature.float().to(x.device).unsqueeze(1)
    greedy = t <= 0
    z = x / torch.where(greedy, torch.ones_like(t), t)
    g = torch.Generator(device=x.device).manual_seed(int(seed) & ((1 << 63) - 1))
    u = torch.rand(x.shape, generator=g, device=x.device).clamp_(1e-12, 1 - 1e-7)
    score = torch.where(greedy, x, z - torch.log(-torch.log(u)))
    tok = score.argmax(-1)
    lp = z.log_softmax(-1).gather(1, tok[:, None]).squeeze(1)
    return tok, lp
