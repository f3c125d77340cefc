"""Multi-process data-parallel tests on CPU (gloo, world size 2): real processes,
real ``build_strategy`` / ``Trainer``, compared against a single-process run
over the union of the ranks' batches (``tests/integration/test_ddp_two_process.py``
of the reference is the model)."""

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

STEPS = 3


def _manifest(strategy: str, out: str):
    from rl_project_b200.core.config import ExperimentManifest

    return ExperimentManifest.from_dict({
        "name": "t", "algorithm": "pretrain", "model_preset": "tiny", "model": {"vocab_size": 64, "block_size": 32},
        "trainer": {"device": "cpu", "precision": {"dtype": "float32"}, "eval_every": 0, "log_every": 0,
                    "max_steps": STEPS, "batch_size": 2, "optimizer": {"learning_rate": 1e-2, "grad_clip": 0.5},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": strategy.replace("_keep", ""), "backend": "gloo", "timeout_s": 120,
                        "reshard_after_forward": not strategy.endswith("_keep")},
        "output_dir": out})


def _global_batches():
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, 64, (4, 33), generator=g) for _ in range(STEPS)]


class _Iter:
    def __init__(self, batches, rows):
        self.batches, self.rows, self.i = batches, rows, 0

    def __iter__(self):
        return self

    def __next__(self):
        b = self.batches[self.i][self.rows]
        self.i += 1
        return b[:, :-1].contiguous(), b[:, 1:].contiguous()


def _train(strategy_name: str, rank: int, world: int, out: str):
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    m = _manifest(strategy_name, os.path.join(out, f"r{rank}"))
    strat = build_strategy(m.distributed) if world > 1 else None
    if strat is not None:
        strat.setup()
    ctx = RunContext.create(m, metrics_backend="none", distributed=False, device_override="cpu")
    torch.manual_seed(0)
    model = TransformerLM(m.model)
    rows = slice(rank * 4 // world, (rank + 1) * 4 // world)
    alg = PretrainAlgorithm(model, _Iter(_global_batches(), rows), PretrainConfig(batch_size=4 // world))
    trainer = Trainer(ctx, alg, strategy=strat)
    losses = [trainer.train_step().loss for _ in range(STEPS)]
    if strat is not None and strategy_name in ("fsdp", "zero2", "fsdp_keep"):
        state = strat.full_state_dict()
    else:
        state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    return losses, state, strat


def _worker(rank, world, port, out, strategy_name):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    losses, state, strat = _train(strategy_name, rank, world, out)
    torch.save({"losses": losses, "state": state}, os.path.join(out, f"result{rank}.pt"))
    strat.teardown()


@pytest.mark.parametrize("strategy_name", ["ddp", "fsdp", "zero2", "fsdp_keep"])  # _keep: no reshard after forward
def test_two_process_matches_single_process(strategy_name):
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(2, free_port(), out, strategy_name), nprocs=2, join=True,
                           start_method="spawn")
        r0 = torch.load(os.path.join(out, "result0.pt"))
        r1 = torch.load(os.path.join(out, "result1.pt"))
        torch.set_num_threads(1)
        single_losses, single_state, _ = _train("single", 0, 1, out)
    # every rank holds the same parameters
    for k in r0["state"]:
        assert torch.allclose(r0["state"][k], r1["state"][k], atol=1e-6), k
    # and they equal the single-process run over the union of the batches
    for k, v in single_state.items():
        if k in r0["state"]:
            assert torch.allclose(r0["state"][k], v, atol=2e-5, rtol=1e-4), (k, (r0["state"][k] - v).abs().max())
    # rank-mean loss equals the single-process loss
    for a, b, s in zip(r0["losses"], r1["losses"], single_losses):
        assert abs((a + b) / 2 - s) < 1e-4
