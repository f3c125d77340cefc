"""Fused reduce-scatter kernel on one GPU: the ranks are emulated as separate
local buffers read through the same pointer table the multi-GPU path uses, and
every flag is raised before the reduce is launched (no kernel waits on another
launch).  Checked against an fp32 PyTorch reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from rl_project_b200.ops._ext import native

    return native()


def _setup(world, shard, slots=2, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bufs = [torch.randn(slots * world * shard, device="cuda", generator=g).bfloat16() for _ in range(world)]
    flags = torch.zeros(slots * world, dtype=torch.int32, device="cuda")
    flag_ptrs = torch.tensor([flags.data_ptr()] * world, dtype=torch.int64, device="cuda")
    return bufs, flags, flag_ptrs


def _ptrs(bufs, slot, world, shard):
    return torch.tensor([b.data_ptr() + slot * world * shard * 2 for b in bufs], dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("world,shard", [(2, 8), (3, 4096), (8, 1 << 16), (12, 200)])
def test_reduce_matches_fp32_reference(world, shard):
    C = _C()
    bufs, flags, flag_ptrs = _setup(world, shard)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for slot, epoch in ((0, 1), (1, 1), (0, 2)):
        for r in range(world):
            C.signal_peers(flag_ptrs, r, slot, epoch)
        ref_full = torch.stack([b[slot * world * shard:(slot + 1) * world * shard].float() for b in bufs]).sum(0)
        ref_full /= world
        for r in range(world):
            out = torch.full((shard,), 0.5, device="cuda")
            sumsq = torch.zeros(1, device="cuda")
            C.fused_reduce_scatter(_ptrs(bufs, slot, world, shard), 0, flags, r, slot, epoch, shard, 1.0 / world,
                                   out, epoch == 2, sumsq, status, int(5e9), 16)
            ref = ref_full[r * shard:(r + 1) * shard] + (0.5 if epoch == 2 else 0.0)
            torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)
            torch.testing.assert_close(sumsq[0], ref.pow(2).sum(), rtol=1e-4, atol=1e-3)
        if epoch == 1:
            for b in bufs:  # refill the slot for the next epoch
                b[slot * world * shard:(slot + 1) * world * shard].normal_()
    assert int(status.item()) == 0


def test_wait_times_out_and_reports():
    """A flag that nothing raises: the bounded wait gives up, sets the status word and writes nothing."""
    C = _C()
    world, shard = 2, 64
    bufs, flags, flag_ptrs = _setup(world, shard)
    C.signal_peers(flag_ptrs, 0, 1, 1)  # rank 1 never signals slot 1
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((shard,), 7.0, device="cuda")
    C.fused_reduce_scatter(_ptrs(bufs, 1, world, shard), 0, flags, 0, 1, 1, shard, 0.5, out, False, None, status,
                           int(2e6), 4)  # 2 ms limit
    torch.cuda.synchronize()
    assert int(status.item()) == (1 | (1 << 8))  # kTimeout on slot 1
    assert bool((out == 7.0).all())
    # the context is still usable and a later, signalled reduce succeeds
    status.zero_()
    C.signal_peers(flag_ptrs, 1, 1, 1)
    C.fused_reduce_scatter(_ptrs(bufs, 1, world, shard), 0, flags, 0, 1, 1, shard, 0.5, out, False, None, status,
                           int(2e9), 4)
    ref = (bufs[0][2 * shard:3 * shard].float() + bufs[1][2 * shard:3 * shard].float()) * 0.5
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)
    assert int(status.item()) == 0
