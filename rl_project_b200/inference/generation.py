"""One prompt in, text out, with throughput statistics (the ``generate_text`` call and stats keys of
``src/forgeline/inference/generation.py``).

The decode runs through the model's cached ``generate`` (or a speculative generator when one is given).
The clock is taken on the host around the call plus the read-back of the tokens, so it covers the device
work; on CUDA the device time between two events on the current stream is reported as well
(``device_s``).
"""

from __future__ import annotations

import time
from typing import Any, Callable, Dict, Optional, Tuple

import torch

from rl_project_b200.core.protocols import GenerationSettings

_DEFAULT = GenerationSettings(max_new_tokens=200, temperature=0.8, top_k=50)


def _decoder(model: Any, s: GenerationSettings, spec_generator: Any) -> Callable[[torch.Tensor], torch.Tensor]:
    if spec_generator is not None:  # speculative decoding takes the subset of settings it supports
        return lambda x: spec_generator.generate(x, max_new_tokens=s.max_new_tokens, temperature=s.temperature,
                                                 top_k=s.top_k)
    return lambda x: model.generate(x, s.max_new_tokens, temperature=s.temperature, top_k=s.top_k, top_p=s.top_p,
                                    min_p=s.min_p, repetition_penalty=s.repetition_penalty, use_cache=s.use_cache,
                                    stop_token_ids=tuple(s.stop_token_ids))


@torch.no_grad()
def generate_text(model: Any, tokenizer: Any, prompt: str, settings: Optional[GenerationSettings] = None,
                  device: Optional[torch.device] = None, spec_generator: Any = None) -> Tuple[str, Dict[str, float]]:
    s = settings or _DEFAULT
    dev = device or next(model.parameters()).device
    prompt_ids = tokenizer.encode(prompt) or [0]  # an empty prompt starts from token 0
    x = torch.tensor([prompt_ids], dtype=torch.long, device=dev)
    run = _decoder(model, s, spec_generator)
    events = None
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
        events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        events[0].record()
    t0 = time.perf_counter()
    y = run(x)
    if events is not None:
        events[1].record()
    out = y[0].tolist()  # the read-back waits for the device
    elapsed = time.perf_counter() - t0
    n_new = len(out) - len(prompt_ids)
    stats: Dict[str, float] = {"n_generated": n_new, "elapsed_s": elapsed,
                               "tokens_per_sec": n_new / elapsed if elapsed > 0 else 0.0}
    if events is not None:
        stats["device_s"] = events[0].elapsed_time(events[1]) / 1e3
    return tokenizer.decode(out), stats
