"""Exact resume of model-parallel runs on two CPU processes (gloo): tensor parallel, pipeline parallel and
expert parallel.  A job trains 4 steps and checkpoints at step 2; a second job (fresh processes) resumes
from that checkpoint.  Every rank must end with bit-identical parameters and step losses, which needs
each rank's own shard, optimizer state, RNG and data position in the checkpoint."""

from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

WORLD = 2
STEPS = 4

MODELS = {
    "tensor_parallel": {"n_layer": 4, "n_head": 4, "n_kv_head": 2, "n_embd": 64},
    "pipeline_parallel": {"n_layer": 4, "n_head": 4, "n_kv_head": 2, "n_embd": 64},
    "expert_parallel": {"n_layer": 2, "use_moe": True, "n_experts": 4, "n_experts_active": 2, "n_shared_experts": 1,
                        "aux_loss_free": True, "score_func": "sigmoid", "bias_update_speed": 0.01,
                        "n_dense_layers": 0},
}


def _manifest(strategy: str, out: str, save_every: int):
    from rl_project_b200.core.config import ExperimentManifest

    sizes = {"tensor_parallel": {"tensor_parallel_size": 2}, "pipeline_parallel": {"pipeline_parallel_size": 2},
             "expert_parallel": {"expert_parallel_size": 2}}[strategy]
    return ExperimentManifest.from_dict({
        "name": strategy, "algorithm": "pretrain", "model_preset": "tiny",
        "model": {"vocab_size": 64, "block_size": 32, **MODELS[strategy]},
        "data": {"kind": "pretraining", "path": "synthetic"},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "eval_every": 0, "log_every": 0,
                    "max_steps": STEPS, "batch_size": 4, "gradient_accumulation_steps": 2, "seed": 5,
                    "optimizer": {"learning_rate": 1e-2, "grad_clip": 0.5},
                    "schedule": {"name": "constant", "warmup_steps": 0},
                    "checkpoint": {"save_every": save_every, "directory": "ckpt", "keep_last": 5}},
        "distributed": {"strategy": strategy, "backend": "gloo", "timeout_s": 120, **sizes},
        "output_dir": out})


def _worker(rank, port, out, strategy, phase):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from rl_project_b200.cli.main import _seed_per_rank
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.core.runtime import seed_everything
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    first = os.path.join(out, "full")
    m = _manifest(strategy, first if phase == "full" else os.path.join(out, "resumed"), 2 if phase == "full" else 0)
    seed_everything(m.trainer.seed)
    strat = build_strategy(m.distributed)
    strat.setup()
    try:
        ctx = RunContext.create(m, metrics_backend="none", distributed=True, device_override="cpu")
        alg = build_algorithm(m, ctx)
        _seed_per_rank(alg, strat, m)
        trainer = Trainer(ctx, alg, strategy=strat)
        if phase == "resumed":
            assert trainer.resume(os.path.join(first, "ckpt", "step_00000002"))
        trainer.fit()
        res = {"losses": [r.loss for r in trainer.history],
               "state": {k: v.detach().clone() for k, v in alg.model.state_dict().items()}}
        ctx.close()
    finally:
        strat.teardown()
    torch.save(res, os.path.join(out, f"{phase}{rank}.pt"))


@pytest.mark.parametrize("strategy", ["tensor_parallel", "pipeline_parallel", "expert_parallel"])
def test_resume_is_exact(tmp_path, strategy):
    out = str(tmp_path)
    for phase in ("full", "resumed"):  # two jobs, each on fresh processes and a fresh rendezvous port
        mp.start_processes(_worker, args=(free_port(), out, strategy, phase), nprocs=WORLD, join=True,
                           start_method="spawn")
    for r in range(WORLD):
        full = torch.load(os.path.join(out, f"full{r}.pt"), weights_only=False)
        res = torch.load(os.path.join(out, f"resumed{r}.pt"), weights_only=False)
        assert res["losses"] == full["losses"][2:], (r, res["losses"], full["losses"])
        for k, v in full["state"].items():
            assert torch.equal(res["state"][k], v), (r, k)
