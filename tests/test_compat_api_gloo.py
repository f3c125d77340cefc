"""Reference-compatible API names: tensor-parallel layers (2 gloo ranks), the 1F1B action list, policy and
allocation helpers."""
import os
import tempfile

import numpy as np
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port


def _tp_worker(rank, port, out):
    import torch.distributed as dist

    from rl_project_b200.parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.manual_seed(0)
    full = torch.nn.Linear(8, 6, bias=True)
    x = torch.randn(3, 8, requires_grad=True)
    ref = full(x)
    col = ColumnParallelLinear.from_linear(full, None, 2, rank)
    col.gather_output = True
    y_col = col(x)
    row = RowParallelLinear.from_linear(full, None, 2, rank)
    y_row = row(x[:, rank * 4:(rank + 1) * 4])
    y_row.sum().backward()
    ok = {"col": float((y_col - ref).abs().max()), "row": float((y_row - ref).abs().max()),
          "row_wgrad_shape": list(row.weight.grad.shape)}
    torch.save(ok, os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_tensor_parallel_layers_equal_the_full_linear():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_tp_worker, args=(free_port(), out), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            res = torch.load(os.path.join(out, f"r{r}.pt"))
            assert res["col"] < 1e-6 and res["row"] < 1e-6 and res["row_wgrad_shape"] == [6, 4]


def test_one_f_one_b_schedule():
    from rl_project_b200.parallel.pipeline import one_f_one_b_schedule

    last = one_f_one_b_schedule(4, 1, 2)
    assert last == [("F", 0), ("B", 0), ("F", 1), ("B", 1), ("F", 2), ("B", 2), ("F", 3), ("B", 3)]
    first = one_f_one_b_schedule(4, 0, 2)
    assert first[0] == ("F", 0) and first[1] == ("F", 1) and first[-1] == ("B", 3)
    assert sorted(first) == sorted(last)


def test_policy_and_allocation_helpers():
    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.domains.allocation.env import StepArrays, StepContext
    from rl_project_b200.models.adapters.lora import apply_lora
    from rl_project_b200.models.policy import has_lora_modules
    from rl_project_b200.models.transformer.model import TransformerLM

    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=64))
    assert not has_lora_modules(m)
    apply_lora(m, rank=2)
    assert has_lora_modules(m)
    a = StepArrays(3, 10, np.array([5.0, 4.0]), 12.0, np.array([1.0, 2.0]), np.array([0.5, 0.6]),
                   np.array([0.7, 0.8]), np.array([0.9, 0.1]))
    c = StepContext.from_arrays(a, 1)
    assert (c.t, c.remaining, c.cum_spend, c.quality) == (3, 4.0, 2.0, 0.1)
    assert StepContext.from_arrays(c.to_arrays()) == c


def _pp_worker(rank, port, out):
    import torch.distributed as dist

    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.pipeline import PipelineScheduler, build_pipeline_stage
    from rl_project_b200.parallel.topology import ParallelMesh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.manual_seed(0)
    model = TransformerLM(model_spec_from_preset("tiny", vocab_size=64, block_size=32))
    g = torch.Generator().manual_seed(3)
    x = torch.randint(0, 64, (4, 32), generator=g)
    y = torch.randint(0, 64, (4, 32), generator=g)
    with torch.no_grad():
        _, ref = model(x, y)
    mesh = ParallelMesh(2, 1, 2, 1, rank).build_groups()
    stage = build_pipeline_stage(model, mesh)
    loss = PipelineScheduler(stage, mesh, n_micro=2).run(x, y)
    grads = sum(float(p.grad.abs().sum()) for p in stage.parameters() if p.grad is not None)
    torch.save({"loss": float(loss), "ref": float(ref), "grads": grads}, os.path.join(out, f"p{rank}.pt"))
    dist.destroy_process_group()


def test_pipeline_scheduler_trains_both_stages():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_pp_worker, args=(free_port(), out), nprocs=2, join=True, start_method="spawn")
        r0, r1 = torch.load(os.path.join(out, "p0.pt")), torch.load(os.path.join(out, "p1.pt"))
    assert abs(r1["loss"] - r1["ref"]) < 1e-4  # last stage: mean loss over the micro-batches
    assert r0["grads"] > 0 and r1["grads"] > 0  # gradients reach the first stage too
