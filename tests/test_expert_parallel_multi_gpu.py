"""Expert parallelism on 2 GPUs against one GPU stepping the concatenated batch (bf16, MLA + MoE).

A 2-layer model of the MLA + MoE configuration (one dense layer, one layer of 64 routed experts with
group-limited top-6 routing, aux-loss-free bias balancing and shared experts).  Rank r of the EP2 run
trains on rows r of each batch and owns half of the experts (peer-memory or NCCL exchange, grouped expert
GEMMs); the single-GPU run trains on every row.  Each rank's loss is a mean over its own tokens, so with
equal token counts the mean of the two ranks' gradients equals the single run's gradient; the router's
expert counts are summed over ranks, so the bias updates agree too.  After three optimizer steps the losses
agree within bf16 tolerance and the updates of the dense parameters agree to 5 % in norm.
"""

from __future__ import annotations

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multi_gpu]
STEPS = 3
ROWS, SEQ = 4, 512


def _batches(vocab: int):
    g = torch.Generator().manual_seed(21)
    return [torch.randint(0, vocab, (ROWS, SEQ + 1), generator=g) for _ in range(STEPS)]


def _run(world: int, rank: int, out: str) -> None:
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    m = ExperimentManifest.from_dict({
        "name": "ep-eq", "algorithm": "pretrain", "model_preset": "bl_mla_moe",
        "model": {"n_layer": 2, "block_size": SEQ},
        "trainer": {"batch_size": ROWS // world, "max_steps": 100, "eval_every": 0, "log_every": 0, "seed": 5,
                    "precision": {"dtype": "bfloat16"},
                    "optimizer": {"learning_rate": 1e-3, "grad_clip": 1.0, "weight_decay": 0.0},
                    "schedule": {"name": "constant", "warmup_steps": 0},
                    "checkpoint": {"save_every": 0, "auto_resume": False}},
        "distributed": {"strategy": "expert_parallel" if world > 1 else "single", "expert_parallel_size": world,
                        "timeout_s": 60},
        "output_dir": os.path.join(out, f"run_{world}_{rank}")})
    strat = build_strategy(m.distributed)
    strat.setup()
    torch.cuda.set_device(rank)
    ctx = RunContext.create(m, metrics_backend="none", distributed=world > 1)
    torch.manual_seed(5)
    with torch.device(ctx.device):
        model = TransformerLM(m.model)
    half = ROWS // world
    rows = slice(rank * half, (rank + 1) * half)
    pool = [b[rows] for b in _batches(m.model.vocab_size)]

    class Data:
        i = 0

        def __iter__(self):
            return self

        def __next__(self):
            b = pool[self.i % STEPS].to(ctx.device)
            self.i += 1
            return b[:, :-1].contiguous(), b[:, 1:].contiguous()

    init = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    alg = PretrainAlgorithm(model, Data(), PretrainConfig(batch_size=half), device=ctx.device)
    trainer = Trainer(ctx, alg, strategy=strat)
    losses = [trainer.train_step().loss for _ in range(STEPS)]
    dense = {k: v.detach().float().cpu() for k, v in model.state_dict().items()
             if ".experts." not in k and "bias" not in k}  # parameters every rank holds in full
    if rank == 0:
        torch.save({"losses": losses, "state": dense, "init": init}, os.path.join(out, f"ep{world}.pt"))
    strat.teardown()


def _worker(rank: int, world: int, port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    _run(world, rank, out)


def test_ep2_equals_one_gpu_on_the_concatenated_batch():
    with tempfile.TemporaryDirectory() as out:
        ctx = mp.get_context("spawn")
        for world in (1, 2):
            port = free_port()
            procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
            for p in procs:
                p.start()
            for p in procs:
                p.join(timeout=900)
                assert p.exitcode == 0
        one, two = torch.load(os.path.join(out, "ep1.pt")), torch.load(os.path.join(out, "ep2.pt"))
        for a, b in zip(one["losses"], two["losses"]):
            assert abs(a - b) < 3e-2 * max(1.0, abs(a)), (one["losses"], two["losses"])
        keys = [k for k in one["state"] if k in two["state"] and k in one["init"]]
        assert keys
        d1 = torch.cat([(one["state"][k] - one["init"][k]).flatten() for k in keys])
        d2 = torch.cat([(two["state"][k] - one["init"][k]).flatten() for k in keys])
        assert (d1 - d2).norm().item() <= 0.05 * d1.norm().item(), ((d1 - d2).norm().item(), d1.norm().item())
