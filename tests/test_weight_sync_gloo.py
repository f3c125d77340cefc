"""Packed parameter broadcast on gloo ranks (host transport): every rank ends with the source's tensors."""
import os
import tempfile

import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port


def _worker(rank, port, out):
    import torch.distributed as dist

    from rl_project_b200.parallel.weight_sync import ParameterBroadcaster

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.manual_seed(rank)
    ts = [torch.randn(37), torch.randn(5, 7), torch.randint(0, 9, (11,))]
    b = ParameterBroadcaster(None, chunk_bytes=64)
    b.broadcast_(ts, src=1)
    torch.save([t.clone() for t in ts], os.path.join(out, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_broadcast_host_transport():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_worker, args=(free_port(), out), nprocs=2, join=True, start_method="spawn")
        a, b = torch.load(os.path.join(out, "r0.pt")), torch.load(os.path.join(out, "r1.pt"))
    torch.manual_seed(1)
    want = [torch.randn(37), torch.randn(5, 7), torch.randint(0, 9, (11,))]
    for x, y, w in zip(a, b, want):
        assert torch.equal(x, w) and torch.equal(y, w)


def test_pieces_cover_every_byte():
    from rl_project_b200.parallel.weight_sync import ParameterBroadcaster

    b = ParameterBroadcaster.__new__(ParameterBroadcaster)
    b.chunk = 48
    ts = [torch.zeros(5), torch.zeros(20), torch.zeros(3)]
    seen = {}
    for chunk in b._pieces(ts):
        assert sum(n for _, _, n in chunk) <= 48
        for v, off, n in chunk:
            seen.setdefault(v.data_ptr(), []).append((off, n))
    assert sorted(sum(n for _, n in v) for v in seen.values()) == [12, 20, 80]
