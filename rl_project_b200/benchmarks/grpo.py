"""GRPO rollout + update throughput (the dense 8B model, 256 prompts x 16 samples,
prompts of 128-512 uniform token ids, up to 1024 generated tokens at temperature 1, last-token-parity
reward, KL 0.04 to a frozen reference), on 1 GPU or N GPUs of one node.

One GRPO step = sample ``prompts x group`` completions with the paged-KV engine, score them, record old and
reference log-probs, and run the clipped GRPO update -- all through the public ``Trainer.train_step``.

* 1 GPU: the policy's own engine generates (prefix sharing: one prefill per prompt).
* N GPUs (``torch.distributed.run``): the learner is this framework's FSDP over all N ranks (gradient
  checkpointing on), and the same ranks form ``N / rollout_tp`` tensor-parallel generation replicas
  (rollouts/replicas.py) refreshed from the learner every step; each rank trains on its share of its
  replica's prompt groups.

Throughput = (prompt + generated tokens of every trajectory trained on, counted from the actual lengths and
summed over ranks) / step time (CUDA events around whole steps, barrier + synchronize on both sides, max
over ranks), after warm-up steps.

    python -m rl_project_b200.benchmarks.grpo --preset bl_dense_1b --prompts 32 --group 16 --max-new 256
    torchrun --nproc-per-node 8 ... -m rl_project_b200.benchmarks.grpo --preset bl_dense_8b --rollout-tp 4
"""

from __future__ import annotations

import argparse
import json
import os
import time
from typing import Any, Dict, List

import torch


def build(args, world: int):
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    distributed = world > 1
    per_rank_prompts = args.prompts // world if distributed else args.prompts
    micro = max(1, per_rank_prompts // args.groups_per_micro)
    rollout = {"group_size": args.group, "max_new_tokens": args.max_new, "temperature": 1.0, "top_p": 1.0,
               "max_prompt_length": args.max_prompt, "engine": "paged"}
    if distributed:
        per_replica = args.prompts * args.group // (world // args.rollout_tp)
        rollout.update(replica_tp=args.rollout_tp, engine_max_batch=min(per_replica, args.engine_batch),
                       engine_kv_blocks=min(per_replica, args.engine_batch) *
                       ((args.max_prompt + args.max_new + 15) // 16 + 1))
    else:
        rollout.update(engine_max_batch=args.prompts * args.group)
    m = ExperimentManifest.from_dict({
        "name": "bench-grpo", "algorithm": "grpo", "model_preset": args.preset,
        "model": ({"n_layer": args.layers} if args.layers else {}),
        "data": {"kind": "verifiable", "path": "synthetic:random_prompts", "seed": 7,
                 "extra": {"n_prompts": max(1024, args.prompts * 4), "min_prompt": args.min_prompt,
                           "max_prompt": args.max_prompt}},
        "reward": {"type": "verifier", "verifier": "last_token_parity"},
        "algorithm_params": {"group_size": args.group, "prompts_per_step": args.prompts, "kl_coef": 0.04,
                             "rollout": rollout},
        "trainer": {"device": args.device, "precision": {"dtype": "bfloat16" if args.device == "cuda" else "float32"},
                    "max_steps": 10 ** 6, "batch_size": per_rank_prompts, "gradient_accumulation_steps": micro,
                    "gradient_checkpointing": bool(distributed or args.grad_ckpt), "eval_every": 0, "log_every": 0,
                    "optimizer": {"learning_rate": 1e-6, "grad_clip": 1.0},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": "fsdp" if distributed else "single", "timeout_s": 900,
                        "backend": "nccl" if args.device == "cuda" else "gloo"},
        "output_dir": "/tmp/rlb_bench_grpo"})
    strategy = build_strategy(m.distributed)
    strategy.setup()
    if args.device == "cuda":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    ctx = RunContext.create(m, metrics_backend="none", distributed=distributed)
    alg = build_algorithm(m, ctx)
    if distributed:
        from rl_project_b200.cli.main import _seed_per_rank

        _seed_per_rank(alg, strategy, m)
    return Trainer(ctx, alg, strategy=strategy), alg, strategy


def _tokens(groups: List[Any]) -> float:
    return float(sum(t.prompt_ids.numel() + t.response_ids.numel() for g in groups for t in g.trajectories))


def run(argv=None) -> Dict[str, Any]:
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="bl_dense_1b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--group", type=int, default=16)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=512)
    ap.add_argument("--max-new", type=int, default=256)
    ap.add_argument("--groups-per-micro", type=int, default=4)
    ap.add_argument("--rollout-tp", type=int, default=4)
    ap.add_argument("--engine-batch", type=int, default=1024, help="sequences a replica decodes at once")
    ap.add_argument("--grad-ckpt", action="store_true")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--device", default="cuda")
    args, _ = ap.parse_known_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    trainer, alg, strategy = build(args, world)
    dist = torch.distributed
    cuda = args.device == "cuda"
    collected: List[Any] = []
    collect_s: List[float] = []
    inner = alg.collect

    def timed_collect(step):  # rollout + rewards + old / reference log-probs
        if cuda:
            torch.cuda.synchronize()
        t = time.perf_counter()
        out = inner(step)
        if cuda:
            torch.cuda.synchronize()
        collect_s.append(time.perf_counter() - t)
        collected.append(out)
        return out

    alg.collect = timed_collect

    def barrier():
        if world > 1:
            dist.barrier()

    def global_max(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if cuda else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def global_sum(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if cuda else "cpu")
        dist.all_reduce(t)
        return float(t.item())

    for _ in range(args.warmup):
        trainer.train_step()
    times, tokens, gen = [], [], []
    for _ in range(args.steps):
        barrier()
        if cuda:
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        t0 = time.perf_counter()
        trainer.train_step()
        if cuda:
            b.record()
            torch.cuda.synchronize()
            dt = a.elapsed_time(b) / 1e3
        else:
            dt = time.perf_counter() - t0
        barrier()
        times.append(global_max(dt))
        groups = collected[-1]
        tokens.append(global_sum(_tokens(groups)))
        gen.append(global_sum(float(sum(t.response_ids.numel() for g in groups for t in g.trajectories))))
    step_s = sum(times) / len(times)
    coll = global_max(sum(collect_s[-args.steps:]) / args.steps)
    out = {"metric": "GRPO rollout+update tokens/s", "value": sum(tokens) / sum(times), "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (uniform token ids, prompt lengths uniform; random-init weights)",
           "generated_tokens_per_s": sum(gen) / sum(times),
           "breakdown": {"collect_ms_max_over_ranks": 1e3 * coll, "update_ms": 1e3 * (step_s - coll)},
           "config": {"model": args.preset + (f" ({args.layers} layers)" if args.layers else ""),
                      "prompts_per_step": args.prompts, "group_size": args.group,
                      "prompt_len": [args.min_prompt, args.max_prompt], "max_new_tokens": args.max_new,
                      "temperature": 1.0, "kl_coef": 0.04, "reward": "last_token_parity",
                      "learner": "fsdp" if world > 1 else "single",
                      "rollout": (f"{world // args.rollout_tp} replicas x TP{args.rollout_tp}, paged-KV continuous "
                                  "batching" if world > 1 else "paged-KV continuous batching"),
                      "tokens_counted": "actual prompt + response lengths of every trajectory trained on"},
           "impl": "ours"}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if hasattr(strategy, "teardown"):
        strategy.teardown()
    return out


def main():
    run()


if __name__ == "__main__":
    main()
