"""The index-error word read at log steps reaches every rank: each rank folds its own code into the
MAX all-reduce that also carries the slowest rank's interval, so a skipped out-of-range index on any
rank (here rank 1 only) is seen by all ranks at the same step.  Two gloo ranks on CPU."""

from __future__ import annotations

import os
import socket
import types

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from rl_project_b200.training.common.trainer import Trainer

        fake = types.SimpleNamespace(strategy=types.SimpleNamespace(world_size=lambda: world),
                                     ctx=types.SimpleNamespace(device=torch.device("cpu")))
        slowest, code = Trainer._slowest_rank_seconds(fake, 0.5 + rank, 7 if rank == 1 else 0)
        clean = Trainer._slowest_rank_seconds(fake, 0.25, 0)
        out.put((rank, slowest, code, clean))
    finally:
        dist.destroy_process_group()


def test_bounds_code_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, slowest, code, clean in got:
        assert slowest == 1.5  # rank 1's interval
        assert code == 7       # rank 1's error word, seen on rank 0 as well
        assert clean == (0.25, 0)


def test_single_process_keeps_its_code():
    from rl_project_b200.training.common.trainer import Trainer

    fake = types.SimpleNamespace(strategy=None, ctx=types.SimpleNamespace(device=torch.device("cpu")))
    assert Trainer._slowest_rank_seconds(fake, 1.0, 3) == (None, 3)
    assert Trainer._bounds_code(fake) == 0  # CPU device: no word to read
