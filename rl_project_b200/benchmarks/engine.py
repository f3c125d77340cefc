"""Inference-engine decode throughput with a per-phase breakdown.

Submits ``prompts x group`` requests (prompt lengths uniform in [min, max];
the ``group`` samples of a prompt share its prefix) and runs the engine to
completion.  Besides aggregate generated tokens/s it reports, per decode step,
the device time of the model's paged decode forward and of sampling (CUDA
events) and the step's host wall time, plus the prefill / decode span totals.

    python -m rl_project_b200.benchmarks.engine --preset bl_dense_1b --prompts 32 --group 16 --max-new 256
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def main():
    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.data.synthetic import random_prompts
    from rl_project_b200.inference import InferenceEngine, SamplingParams
    from rl_project_b200.models.transformer.model import TransformerLM

    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="bl_dense_1b")
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--group", type=int, default=16)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=512)
    ap.add_argument("--max-new", type=int, default=256)
    ap.add_argument("--temperature", type=float, default=1.0)
    args = ap.parse_args()
    torch.manual_seed(0)
    spec = model_spec_from_preset(args.preset)
    with torch.device("cuda"):
        model = TransformerLM(spec).to(torch.bfloat16).eval()
    n = args.prompts * args.group
    per_seq = (args.max_prompt + args.max_new + 15) // 16 + 1
    eng = InferenceEngine(model, max_batch=n, max_blocks=n * per_seq, profile=True)
    prompts = random_prompts(args.prompts, spec.vocab_size, args.min_prompt, args.max_prompt, seed=1)
    params = SamplingParams(max_tokens=args.max_new, temperature=args.temperature, top_k=None)
    eng.generate_batch([prompts[0].tolist()], SamplingParams(max_tokens=4, temperature=1.0, top_k=None))  # warm-up
    eng.reset_profile()
    eng.tracer = type(eng.tracer)()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    reqs = eng.generate_batch([p.tolist() for p in prompts for _ in range(args.group)], params)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    gen = sum(len(r.generated_tokens) for r in reqs)
    print(json.dumps({"metric": "engine generated tokens/s", "value": gen / wall, "unit": "tokens/s",
                      "sequences": n, "generated_tokens": gen, "wall_s": wall, "config": vars(args),
                      "per_decode_step_ms": eng.profile_summary(),
                      "spans_ms": {k: round(v["total_ms"], 1) for k, v in eng.tracer.summary().items()}}),
          flush=True)


if __name__ == "__main__":
    main()
