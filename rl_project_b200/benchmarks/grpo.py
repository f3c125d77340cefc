"""GRPO rollout + update throughput (the GRPO benchmark shape -- 8B, 256 prompts x 16 -- scaled by flags).

One GRPO step = sample ``prompts x group`` completions with the paged-KV
inference engine (prefix sharing: one prefill per prompt), score them with the
last-token-parity verifier, record old and reference log-probs, and run the
clipped GRPO update with KL to a frozen reference copy -- all through the
public ``Trainer.train_step``.  Throughput = (prompt + generated tokens of
every trajectory) / step time, timed with CUDA events around whole steps
(synchronised on both sides) after warm-up steps.  Prompts are uniform token
ids with lengths uniform in [min_prompt, max_prompt]; weights are random.

    python -m rl_project_b200.benchmarks.grpo --preset bl_dense_1b --prompts 32 --group 16 --max-new 256
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def build(args):
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    micro = max(1, args.prompts // args.groups_per_micro)
    m = ExperimentManifest.from_dict({
        "name": "bench-grpo", "algorithm": "grpo", "model_preset": args.preset,
        "data": {"kind": "verifiable", "path": "synthetic:random_prompts", "seed": 7,
                 "extra": {"n_prompts": max(1024, args.prompts * 4), "min_prompt": args.min_prompt,
                           "max_prompt": args.max_prompt}},
        "reward": {"type": "verifier", "verifier": "last_token_parity"},
        "algorithm_params": {"group_size": args.group, "prompts_per_step": args.prompts, "kl_coef": 0.04,
                             "rollout": {"group_size": args.group, "max_new_tokens": args.max_new,
                                         "temperature": 1.0, "top_p": 1.0, "max_prompt_length": args.max_prompt,
                                         "engine": "paged", "engine_max_batch": args.prompts * args.group}},
        "trainer": {"device": args.device, "precision": {"dtype": "bfloat16" if args.device == "cuda" else "float32"}, "max_steps": 10 ** 6,
                    "batch_size": args.prompts, "gradient_accumulation_steps": micro, "eval_every": 0,
                    "log_every": 0, "optimizer": {"learning_rate": 1e-6, "grad_clip": 1.0},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "output_dir": "/tmp/rlb_bench_grpo"})
    ctx = RunContext.create(m, metrics_backend="none")
    alg = build_algorithm(m, ctx)
    return Trainer(ctx, alg), alg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="bl_dense_1b")
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--group", type=int, default=16)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=512)
    ap.add_argument("--max-new", type=int, default=256)
    ap.add_argument("--groups-per-micro", type=int, default=4)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--device", default="cuda")
    args = ap.parse_args()
    trainer, alg = build(args)
    collect_s: list = []
    inner_collect = alg.collect

    def timed_collect(step):  # rollout + rewards + old / reference log-probs, timed on the device
        if args.device == "cuda":
            torch.cuda.synchronize()
        t = time.perf_counter()
        out = inner_collect(step)
        if args.device == "cuda":
            torch.cuda.synchronize()
        collect_s.append(time.perf_counter() - t)
        return out

    alg.collect = timed_collect
    for _ in range(args.warmup):
        trainer.train_step()
    times, tokens, gen_tokens, rollout_s = [], [], [], []
    cuda = args.device == "cuda"
    for _ in range(args.steps):
        if cuda:
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        t0 = time.perf_counter()
        res = trainer.train_step()
        if cuda:
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) / 1e3)
        else:
            times.append(time.perf_counter() - t0)
        eng = alg.rollouts.inference_engine()
        st = eng.stats() if eng is not None else {}
        rl = res.metrics.get("response_len", 0.0)
        n = args.prompts * args.group
        gen_tokens.append(rl * n)
        plen = (args.min_prompt + args.max_prompt) / 2  # expected prompt length of the uniform draw
        tokens.append(n * (rl + plen))
        rollout_s.append(st.get("spans", {}).get("decode", {}).get("total_ms", 0.0) / 1e3)
    step_s = sum(times) / len(times)
    coll = collect_s[-args.steps:]
    breakdown = {"collect_ms": 1e3 * sum(coll) / len(coll), "update_ms": 1e3 * (step_s - sum(coll) / len(coll))}
    out = {"metric": "GRPO rollout+update tokens/s", "value": sum(tokens) / sum(times), "unit": "tokens/s",
           "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
           "generated_tokens_per_s": sum(gen_tokens) / sum(times), "breakdown": breakdown, "dtype": "bf16",
           "data": "synthetic (uniform token ids, prompt lengths uniform; random-init weights)",
           "config": {"model": args.preset, "prompts_per_step": args.prompts, "group_size": args.group,
                      "prompt_len": [args.min_prompt, args.max_prompt], "max_new_tokens": args.max_new,
                      "temperature": 1.0, "kl_coef": 0.04, "engine": "paged-KV continuous batching",
                      "reward": "last_token_parity"},
           "engine": {k: v for k, v in (alg.rollouts.inference_engine().stats().items()
                                        if alg.rollouts.inference_engine() else []) if k != "spans"}}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
