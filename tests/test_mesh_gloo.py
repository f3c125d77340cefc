"""Tensor / pipeline / 3-D parallel training on CPU gloo ranks against one process.

Each mesh run trains the same model on the same global batches as a single
process; the losses must agree step by step and the TP shards / PP stages must
reassemble into the single-process parameters.
"""
from __future__ import annotations

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

STEPS = 3
ROWS = 8


def _manifest(tp: int, pp: int, out: str, micro: int):
    from rl_project_b200.core.config import ExperimentManifest

    strategy = "hybrid" if tp > 1 and pp > 1 else ("tensor_parallel" if tp > 1 else
                                                    ("pipeline_parallel" if pp > 1 else "single"))
    return ExperimentManifest.from_dict({
        "name": "mesh", "algorithm": "pretrain", "model_preset": "tiny",
        "model": {"vocab_size": 64, "block_size": 32, "n_layer": 4, "n_head": 4, "n_kv_head": 2, "n_embd": 64},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "eval_every": 0, "log_every": 0,
                    "max_steps": STEPS, "batch_size": 2, "gradient_accumulation_steps": micro,
                    "optimizer": {"learning_rate": 1e-2, "grad_clip": 0.5},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": strategy, "backend": "gloo", "tensor_parallel_size": tp,
                        "pipeline_parallel_size": pp, "timeout_s": 30},
        "output_dir": out})


def _batches():
    g = torch.Generator().manual_seed(11)
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


def _train(tp, pp, world, rank, out, micro):
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    m = _manifest(tp, pp, os.path.join(out, f"r{rank}"), micro)
    strat = None
    dp_rank, dp = 0, 1
    if world > 1:
        strat = build_strategy(m.distributed)
        strat.setup()
        dp_rank, dp = strat.mesh.dp_rank, strat.mesh.dp_size
    ctx = RunContext.create(m, metrics_backend="none", distributed=False, device_override="cpu")
    torch.manual_seed(0)
    model = TransformerLM(m.model)
    rows = slice(dp_rank * ROWS // dp, (dp_rank + 1) * ROWS // dp)
    alg = PretrainAlgorithm(model, _Iter(_batches(), rows), PretrainConfig(batch_size=ROWS // dp))
    trainer = Trainer(ctx, alg, strategy=strat)
    losses = [trainer.train_step().loss for _ in range(STEPS)]
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    coords = strat.mesh.coords() if strat is not None else {"tp": 0, "pp": 0, "dp": 0}
    return losses, state, coords, strat


def _worker(rank, world, port, out, tp, pp, micro):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    losses, state, coords, strat = _train(tp, pp, world, rank, out, micro)
    torch.save({"losses": losses, "state": state, "coords": coords}, os.path.join(out, f"result{rank}.pt"))
    strat.teardown()


ROW_SPLIT = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "w1.weight", "w3.weight")
COL_SPLIT = ("attn.c_proj.weight", "w2.weight")


def _reassemble(results, tp):
    """Full parameters from the shards of dp replica 0."""
    full = {}
    by_tp = {}
    for r in results:
        if r["coords"]["dp"] != 0:
            continue
        for k, v in r["state"].items():
            by_tp.setdefault(k, {})[r["coords"]["tp"]] = v
    for k, parts in by_tp.items():
        ordered = [parts[t] for t in sorted(parts)]
        if tp > 1 and k.endswith(ROW_SPLIT):
            full[k] = torch.cat(ordered, 0)
        elif tp > 1 and k.endswith(COL_SPLIT):
            full[k] = torch.cat(ordered, 1)
        else:
            full[k] = ordered[0]
    return full


@pytest.mark.parametrize("tp,pp,world,micro", [(2, 1, 2, 1), (1, 2, 2, 2), (2, 2, 4, 2), (1, 2, 4, 4)])
def test_mesh_matches_single_process(tp, pp, world, micro):
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(world, free_port(), out, tp, pp, micro), nprocs=world, join=True,
                           start_method="spawn")
        results = [torch.load(os.path.join(out, f"result{r}.pt")) for r in range(world)]
        torch.set_num_threads(1)
        single_losses, single_state, _, _ = _train(1, 1, 1, 0, out, 1)
    dp = world // (tp * pp)
    for step in range(STEPS):  # the mean over data-parallel replicas equals the single-process loss
        mean = sum(r["losses"][step] for r in results if r["coords"]["tp"] == 0 and
                   r["coords"]["pp"] == 0) / dp
        assert abs(mean - single_losses[step]) < 2e-4, (step, mean, single_losses[step])
    full = _reassemble(results, tp)
    assert set(full) >= {k for k in single_state if ".h." in k}
    for k, v in single_state.items():
        if k in full:
            # Adam turns fp32 reduction-order noise on near-zero gradients into small update differences:
            # bound the worst element loosely and the overall difference tightly
            d = (full[k] - v).abs()
            assert d.max() < 5e-4 and d.norm() / v.norm() < 1e-4, (k, d.max(), d.norm() / v.norm())
