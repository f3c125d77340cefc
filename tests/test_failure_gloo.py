"""Failure detection on the host (gloo ranks, no GPU): a rank that dies, a rank that leaves, a rank
that never joins, a message that never arrives -- the survivors get a typed error instead of hanging."""
import os
import tempfile
import time

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port


def _init(rank, world, port, timeout_s=30.0):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _dead_rank_worker(rank, port, out, mode):
    import torch.distributed as dist

    from rl_project_b200.core.errors import DistributedTimeoutError
    from rl_project_b200.parallel.health import monitor_for_process_group

    _init(rank, 3, port)
    mon = monitor_for_process_group(interval_s=0.1, timeout_s=1.0)
    mon.wait_all_alive(10.0)
    dist.barrier()
    if rank == 2:
        if mode == "leave":
            mon.stop("preempted")
            time.sleep(5.0)  # stay alive (the store lives in rank 0's process) but silent
        else:
            mon._stop.set()  # heartbeat thread stops as if the process had frozen
            time.sleep(5.0)
        os._exit(0)  # no clean shutdown of the process group
    msg = ""
    t0 = time.monotonic()
    while time.monotonic() - t0 < 15.0:
        try:
            mon.check()
        except DistributedTimeoutError as e:
            msg = str(e)
            break
        time.sleep(0.05)
    with open(os.path.join(out, f"r{rank}.txt"), "w") as fh:
        fh.write(f"{msg}\n{time.monotonic() - t0:.2f}")
    time.sleep(6.0 if rank == 0 else 0.0)  # rank 0 hosts the store: outlive the others
    os._exit(0)


@pytest.mark.parametrize("mode", ["crash", "leave"])
def test_gone_rank_is_reported(mode):
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_dead_rank_worker, args=(free_port(), out, mode), nprocs=3, join=True,
                           start_method="spawn")
        for r in (0, 1):
            msg, took = open(os.path.join(out, f"r{r}.txt")).read().split("\n")
            assert "rank 2" in msg, msg
            assert ("left: preempted" in msg) if mode == "leave" else ("no heartbeat" in msg), msg
            assert float(took) < 10.0


def _never_joins():
    from rl_project_b200.parallel.runtime import init_process_group

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port()), RANK="0", WORLD_SIZE="2")
    init_process_group("gloo", timeout_s=3.0)


def test_rank_that_never_joins_times_out():
    t0 = time.monotonic()
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_never_joins)
    p.start()
    p.join(60)
    alive = p.is_alive()
    if alive:
        p.kill()
    assert not alive and p.exitcode != 0  # init raised (process group timeout), it did not hang
    assert time.monotonic() - t0 < 60


def _lost_message_worker(rank, port, out):
    import torch.distributed as dist

    _init(rank, 2, port, timeout_s=3.0)
    if rank == 0:
        buf = torch.zeros(4)
        t0 = time.monotonic()
        err = ""
        try:
            dist.recv(buf, src=1)  # rank 1 never sends: the message is lost
        except Exception as e:  # gloo raises after the group timeout
            err = type(e).__name__
        with open(os.path.join(out, "r0.txt"), "w") as fh:
            fh.write(f"{err}\n{time.monotonic() - t0:.2f}")
    else:
        time.sleep(6.0)
    os._exit(0)


def test_lost_message_ends_with_timeout():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_lost_message_worker, args=(free_port(), out), nprocs=2, join=True, start_method="spawn")
        err, took = open(os.path.join(out, "r0.txt")).read().split("\n")
    assert err and float(took) < 30.0
