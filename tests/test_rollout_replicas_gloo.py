"""Tensor-parallel rollout replicas (rollouts/replicas.py) on two CPU processes (gloo).

1. A TP=2 replica synced from a full model reproduces the full model's prompt logits, and both ranks of
   the replica sample the same completions (the all-reduced logits and the sampler seeds agree).
2. GRPO with an FSDP learner and one TP=2 rollout replica runs through the factory and the Trainer:
   both ranks train on their own half of the replica's prompt groups, losses are finite and the learner's
   weights move.
"""

from __future__ import annotations

import math
import os

import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

WORLD = 2


def _env(rank: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)


def _replica_worker(rank: int, port: int, q) -> None:
    _env(rank, port)
    import torch.distributed as dist

    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.inference.requests import SamplingParams
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.rollouts.replicas import RolloutReplicas

    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        spec = model_spec_from_preset("tiny", vocab_size=97, block_size=64)
        torch.manual_seed(0)
        full = TransformerLM(spec).eval()
        rep = RolloutReplicas(spec, 2, torch.device("cpu"), torch.float32, max_batch=8, max_blocks=64)
        rep.sync_from_module(full)
        ids = torch.randint(0, 97, (3, 20), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            ref, _ = full.prefill(ids)
            got, _ = rep.model.prefill(ids)
        err = (ref - got).abs().max().item()
        outs = rep.generate([[1, 2, 3, 4], [5, 6, 7]], 3, SamplingParams(max_tokens=6, temperature=1.0), seed=11)
        q.put((rank, err, outs, rep.replica, rep.tp_rank))
    finally:
        dist.destroy_process_group()


def test_tp_replica_matches_full_model_and_ranks_agree():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_replica_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, e0, o0, rp0, t0), (r1, e1, o1, rp1, t1) = res
    assert e0 < 1e-4 and e1 < 1e-4  # the sharded copy computes the full model's logits
    assert (rp0, t0, rp1, t1) == (0, 0, 0, 1)  # one replica of two ranks
    assert o0 == o1  # identical completions on both ranks of the replica
    assert [len(g) for g in o0] == [3, 3] and all(1 <= len(c) <= 6 for g in o0 for c in g)


def _grpo_worker(rank: int, port: int, out: str, q) -> None:
    _env(rank, port)
    from rl_project_b200.cli.main import _seed_per_rank
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.core.runtime import seed_everything
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    m = ExperimentManifest.from_dict({
        "name": "grpo-replicas", "algorithm": "grpo", "model_preset": "tiny",
        "model": {"vocab_size": 64, "block_size": 64},
        "data": {"kind": "verifiable", "path": "synthetic:random_prompts", "seed": 5,
                 "extra": {"n_prompts": 32, "min_prompt": 4, "max_prompt": 12}},
        "reward": {"type": "verifier", "verifier": "last_token_parity"},
        "algorithm_params": {"group_size": 4, "prompts_per_step": 4, "kl_coef": 0.04,
                             "rollout": {"group_size": 4, "max_new_tokens": 6, "temperature": 1.0,
                                         "max_prompt_length": 12, "engine": "paged", "engine_max_batch": 32,
                                         "engine_kv_blocks": 64, "replica_tp": 2}},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": 2, "batch_size": 4,
                    "eval_every": 0, "log_every": 1, "seed": 3,
                    "optimizer": {"learning_rate": 1e-2, "grad_clip": 1.0},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": "fsdp", "backend": "gloo", "timeout_s": 120},
        "output_dir": out})
    seed_everything(m.trainer.seed)
    strategy = build_strategy(m.distributed)
    strategy.setup()
    try:
        ctx = RunContext.create(m, metrics_backend="none", distributed=True, device_override="cpu")
        alg = build_algorithm(m, ctx)
        _seed_per_rank(alg, strategy, m)
        trainer = Trainer(ctx, alg, strategy=strategy)
        w0 = torch.cat([v.flatten() for _, v in sorted(strategy.full_state_dict().items())])
        trainer.fit()
        w1 = torch.cat([v.flatten() for _, v in sorted(strategy.full_state_dict().items())])
        groups = alg.collect(99)  # this rank's share of one more step's groups
        q.put((rank, [r.loss for r in trainer.history], float((w1 - w0).abs().max()), len(groups),
               [len(g.trajectories) for g in groups]))
        ctx.close()
    finally:
        strategy.teardown()


def test_grpo_with_fsdp_learner_and_tp_rollout_replica(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_grpo_worker, args=(r, port, str(tmp_path), q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=400) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, losses, moved, n_groups, sizes in res:
        assert len(losses) == 2 and all(math.isfinite(x) for x in losses)
        assert moved > 0  # the learner updated
        assert n_groups == 2 and sizes == [4, 4]  # half of the replica's 4 prompt groups, 4 samples each
