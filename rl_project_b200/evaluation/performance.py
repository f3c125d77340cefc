"""Generation latency / throughput / memory measurement.

``measure_generation`` keeps the reference's metric keys
(``src/forgeline/evaluation/performance.py:14-50``) and times each run with CUDA
events on the launching stream (synchronised on both sides) on a GPU, with the
host clock on CPU.  ``measure_engine`` measures the continuous-batching
inference engine: many concurrent requests, aggregate generated tokens/s.
"""

from __future__ import annotations

import statistics
import time
from typing import Any, Dict, List, Optional, Sequence

import torch

from rl_project_b200.core.protocols import EvaluationResult, GenerationSettings


class _Timer:
    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self.device = device

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize(self.device)
            self.a, self.b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self.a.record()
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.cuda:
            self.b.record()
            torch.cuda.synchronize(self.device)
            self.seconds = self.a.elapsed_time(self.b) / 1e3
        else:
            self.seconds = time.perf_counter() - self.t0
        return False


def measure_generation(policy, prompt_ids: torch.Tensor, max_new_tokens: int = 32, runs: int = 3, warmup: int = 1,
                       temperature: float = 0.0) -> Dict[str, float]:
    settings = GenerationSettings(max_new_tokens=max_new_tokens, temperature=temperature)
    device = policy.device
    ids = (prompt_ids.unsqueeze(0) if prompt_ids.dim() == 1 else prompt_ids).to(device)
    for _ in range(warmup):
        policy.generate(ids, settings)
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)
    latencies: List[float] = []
    tokens: List[int] = []
    for _ in range(runs):
        with _Timer(device) as t:
            out = policy.generate(ids, settings)
        latencies.append(t.seconds)
        tokens.append(int(out.shape[0] * out.shape[1]))
    total_time = sum(latencies)
    metrics = {"tokens_per_second": sum(tokens) / total_time if total_time > 0 else 0.0,
               "latency_mean_s": statistics.mean(latencies), "latency_p50_s": statistics.median(latencies),
               "latency_max_s": max(latencies), "tokens_generated": float(sum(tokens)), "runs": float(runs)}
    if device.type == "cuda":
        metrics["peak_memory_gb"] = torch.cuda.max_memory_allocated(device) / 1e9
    return metrics


def measure_engine(engine, prompts: Sequence[Sequence[int]], params: Any, warmup: bool = True) -> Dict[str, float]:
    """Submit every prompt at once and run the engine until idle; aggregate generated tokens/s."""
    if warmup:
        engine.generate_batch([list(prompts[0])], params)
    device = engine.device
    before = engine.decode_steps
    with _Timer(device) as t:
        reqs = engine.generate_batch([list(p) for p in prompts], params)
    gen = sum(len(r.generated_tokens) for r in reqs)
    lat = sorted(r.latency_s for r in reqs if r.latency_s is not None)
    return {"tokens_per_second": gen / t.seconds if t.seconds > 0 else 0.0, "tokens_generated": float(gen),
            "requests": float(len(reqs)), "seconds": t.seconds, "decode_steps": float(engine.decode_steps - before),
            "latency_p50_s": lat[len(lat) // 2] if lat else 0.0,
            "latency_p95_s": lat[min(len(lat) - 1, int(len(lat) * 0.95))] if lat else 0.0}


class PerformanceSuite:
    name = "performance"

    def __init__(self, prompt_ids: torch.Tensor, max_new_tokens: int = 32, runs: int = 3):
        self.prompt_ids, self.max_new_tokens, self.runs = prompt_ids, max_new_tokens, runs

    def run(self, policy, **kwargs: Any) -> EvaluationResult:
        m = measure_generation(policy, self.prompt_ids, self.max_new_tokens, self.runs)
        return EvaluationResult(self.name, m, n_samples=self.runs, details={"device": str(policy.device)})
