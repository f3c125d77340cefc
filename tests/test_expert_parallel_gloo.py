"""Expert parallelism on CPU gloo ranks against one process (same model, same data)."""
from __future__ import annotations

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

STEPS = 3
ROWS = 4


def _manifest(world: int, out: str):
    from rl_project_b200.core.config import ExperimentManifest

    return ExperimentManifest.from_dict({
        "name": "ep", "algorithm": "pretrain", "model_preset": "tiny",
        "model": {"vocab_size": 64, "block_size": 32, "n_layer": 2, "use_moe": True, "n_experts": 4,
                  "n_experts_active": 2, "n_shared_experts": 1, "aux_loss_free": True, "score_func": "sigmoid",
                  "bias_update_speed": 0.01, "n_dense_layers": 0},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "eval_every": 0, "log_every": 0,
                    "max_steps": STEPS, "batch_size": 2, "optimizer": {"learning_rate": 1e-2, "grad_clip": 0.5},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": "expert_parallel" if world > 1 else "single", "backend": "gloo",
                        "expert_parallel_size": max(world, 1), "timeout_s": 30},
        "output_dir": out})


def _batches():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 64, (ROWS, 17), generator=g) for _ in range(STEPS)]


class _Iter:
    def __init__(self, batches, rows):
        self.batches, self.rows, self.i = batches, rows, 0

    def __iter__(self):
        return self

    def __next__(self):
        b = self.batches[self.i][self.rows]
        self.i += 1
        return b[:, :-1].contiguous(), b[:, 1:].contiguous()


def _train(world, rank, out):
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    m = _manifest(world, os.path.join(out, f"r{rank}"))
    strat = None
    if world > 1:
        strat = build_strategy(m.distributed)
        strat.setup()
    ctx = RunContext.create(m, metrics_backend="none", distributed=False, device_override="cpu")
    torch.manual_seed(0)
    model = TransformerLM(m.model)
    rows = slice(rank * ROWS // world, (rank + 1) * ROWS // world)
    alg = PretrainAlgorithm(model, _Iter(_batches(), rows), PretrainConfig(batch_size=ROWS // world))
    trainer = Trainer(ctx, alg, strategy=strat)
    losses = [trainer.train_step().loss for _ in range(STEPS)]
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    return losses, state, strat


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    losses, state, strat = _train(world, rank, out)
    torch.save({"losses": losses, "state": state}, os.path.join(out, f"result{rank}.pt"))
    strat.teardown()


def test_expert_parallel_matches_single_process():
    world = 2
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(world, free_port(), out), nprocs=world, join=True, start_method="spawn")
        res = [torch.load(os.path.join(out, f"result{r}.pt")) for r in range(world)]
        torch.set_num_threads(1)
        single_losses, single_state, _ = _train(1, 0, out)
    for s in range(STEPS):
        assert abs(sum(r["losses"][s] for r in res) / world - single_losses[s]) < 2e-4
    merged = {}
    for r in res:
        merged.update(r["state"])
    for k, v in single_state.items():
        assert k in merged, k
        d = (merged[k] - v).abs()
        assert d.max() < 5e-4 and d.norm() / (v.norm() + 1e-12) < 1e-4, (k, d.max())
    # experts live on one rank each; router biases are identical everywhere
    assert "transformer.h.0.ffn.experts.0.w1.weight" in res[0]["state"]
    assert "transformer.h.0.ffn.experts.0.w1.weight" not in res[1]["state"]
    assert torch.equal(res[0]["state"]["transformer.h.0.ffn.gate.expert_bias"],
                       res[1]["state"]["transformer.h.0.ffn.gate.expert_bias"])
