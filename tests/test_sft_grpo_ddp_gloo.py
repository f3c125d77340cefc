"""Tiny SFT (DDP and FSDP) -> GRPO (DDP) on two CPU processes (gloo), through the manifest,
the algorithm factory, ``build_strategy`` and ``Trainer`` as ``forgeline-b200 train``
runs them.

Checks: replicas hold identical weights after every phase while the ranks see
different data; losses are finite; a run resumed from the middle checkpoint ends
bit-identical to the uninterrupted run on every rank (each rank restores its own
RNG and data position); GRPO reward rises from the SFT checkpoint.  The
reference's ``tests/integration/test_ddp_two_process.py:17-81`` covers the same
replica check for pretraining and GRPO.
"""

from __future__ import annotations

import math
import os

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

WORLD = 2


def _manifest(alg: str, out: str, steps: int, strategy: str = "ddp", **extra):
    from rl_project_b200.core.config import ExperimentManifest

    data = {"kind": "supervised" if alg == "sft" else "verifiable", "path": "synthetic:addition",
            "tokenizer": "byte", "max_length": 32, "extra": {"n_tasks": 64}}
    return ExperimentManifest.from_dict({
        "name": alg, "algorithm": alg, "model_preset": "tiny", "model": {"vocab_size": 256, "block_size": 64},
        "data": data,
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "max_steps": steps, "batch_size": 4,
                    "eval_every": 0, "log_every": 1, "seed": 3,
                    "optimizer": {"learning_rate": extra.pop("lr", 3e-3), "grad_clip": 1.0},
                    "schedule": {"name": "constant", "warmup_steps": 0},
                    "checkpoint": {"save_every": extra.pop("save_every", 0), "directory": "ckpt", "keep_last": 5}},
        "distributed": {"strategy": strategy, "backend": "gloo", "timeout_s": 120},
        "output_dir": out, **extra})


def _run(manifest, resume=None):
    """One phase on this rank; returns (per-step losses, metrics, flat parameters)."""
    from rl_project_b200.cli.main import _seed_per_rank
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.core.runtime import seed_everything
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    seed_everything(manifest.trainer.seed)
    strategy = build_strategy(manifest.distributed)
    strategy.setup()
    try:
        ctx = RunContext.create(manifest, metrics_backend="none", distributed=True, device_override="cpu")
        alg = build_algorithm(manifest, ctx)
        _seed_per_rank(alg, strategy, manifest)
        trainer = Trainer(ctx, alg, strategy=strategy)
        if resume:
            assert trainer.resume(resume)
        trainer.fit()
        losses = [r.loss for r in trainer.history]
        metrics = [dict(r.metrics) for r in trainer.history]
        if strategy.name in ("fsdp", "zero2"):  # the full fp32 weights (collective)
            flat = torch.cat([v.flatten() for _, v in sorted(strategy.full_state_dict().items())])
        else:
            flat = torch.cat([p.detach().flatten().clone() for p in trainer.params])
        ctx.close()
    finally:
        strategy.teardown()
    return losses, metrics, flat


def _worker(rank, port, out, phase):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    if phase.startswith("sft"):
        strategy = "fsdp" if "fsdp" in phase else "ddp"
        first = phase.replace("_resumed", "")
        if phase.endswith("_resumed"):  # a new job resuming the first one's middle checkpoint
            res = _run(_manifest("sft", os.path.join(out, phase), 6, strategy),
                       resume=os.path.join(out, first, "ckpt", "step_00000003"))
        else:
            res = _run(_manifest("sft", os.path.join(out, phase), 6, strategy, save_every=3))
    else:
        resumed = phase == "grpo_resumed"
        res = _run(_manifest("grpo", os.path.join(out, phase), 24, lr=3e-2, save_every=0 if resumed else 12,
                             checkpoint_path=os.path.join(out, "sft", "ckpt", "final"),
                             reward={"type": "verifier", "verifier": "last_token_parity"},
                             algorithm_params={"group_size": 4, "prompts_per_step": 2, "kl_coef": 0.0,
                                               "rollout": {"max_new_tokens": 6, "temperature": 1.0}}),
                   resume=os.path.join(out, "grpo", "ckpt", "step_00000012") if resumed else None)
    torch.save(res, os.path.join(out, f"{phase}{rank}.pt"))


def _phase(out, phase):
    """One job: WORLD fresh processes on a fresh rendezvous port."""
    mp.start_processes(_worker, args=(free_port(), out, phase), nprocs=WORLD, join=True, start_method="spawn")
    return [torch.load(os.path.join(out, f"{phase}{r}.pt"), weights_only=False) for r in range(WORLD)]


@pytest.fixture(scope="module")
def runs(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("ddp_sft_grpo"))
    return {ph: _phase(out, ph) for ph in ("sft", "sft_resumed", "grpo", "grpo_resumed", "sft_fsdp",
                                           "sft_fsdp_resumed")}


@pytest.mark.parametrize("job", ["sft", "sft_fsdp"])
def test_sft_replicas_identical_and_finite(runs, job):
    (l0, _, w0), (l1, _, w1) = runs[job]
    assert torch.equal(w0, w1)
    assert len(l0) == 6 and all(math.isfinite(x) for x in l0 + l1)
    assert l0 != l1  # the ranks trained on different batches


@pytest.mark.parametrize("job", ["sft", "sft_fsdp"])
def test_sft_resume_is_exact_on_every_rank(runs, job):
    for r in range(WORLD):
        full_losses, _, w_full = runs[job][r]
        res_losses, _, w_res = runs[f"{job}_resumed"][r]
        assert res_losses == full_losses[3:], (r, res_losses, full_losses)
        assert torch.equal(w_res, w_full), r


def test_grpo_replicas_identical_and_reward_rises(runs):
    (l0, m0, w0), (l1, m1, w1) = runs["grpo"]
    assert torch.equal(w0, w1)
    assert all(math.isfinite(x) for x in l0 + l1)
    reward = [(a["reward_mean"] + b["reward_mean"]) / 2 for a, b in zip(m0, m1)]
    first, last = sum(reward[:8]) / 8, sum(reward[-8:]) / 8
    assert last > first + 0.15, reward


def test_grpo_resume_is_exact_on_every_rank(runs):
    """Prompt choice, sampled rollouts and updates after the step-12 checkpoint repeat exactly."""
    for r in range(WORLD):
        full_losses, _, w_full = runs["grpo"][r]
        res_losses, _, w_res = runs["grpo_resumed"][r]
        assert res_losses == full_losses[12:], (r, res_losses, full_losses[12:])
        assert torch.equal(w_res, w_full), r
