"""Paged-KV decode attention kernels against an fp32 PyTorch reference."""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

BLOCK = 16


def _reference(q, k_pool, v_pool, tables, lens, scale, softcap, window):
    B, Hq, D = q.shape
    Hkv = k_pool.shape[1]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, D, device=q.device)
    for b in range(B):
        n = int(lens[b])
        blocks = tables[b, : (n + BLOCK - 1) // BLOCK].long()
        k = k_pool[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :n].float()
        v = v_pool[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :n].float()
        k = k.repeat_interleave(G, 0)
        v = v.repeat_interleave(G, 0)
        s = torch.einsum("hd,htd->ht", q[b].float(), k) * scale
        if softcap > 0:
            s = torch.tanh(s / softcap) * softcap
        if window > 0 and n > window:
            s[:, : n - window] = float("-inf")
        out[b] = torch.einsum("ht,htd->hd", s.softmax(-1), v)
    return out


@pytest.mark.parametrize("Hq,Hkv,D", [(8, 2, 128), (4, 4, 64), (16, 2, 64), (4, 1, 32)])
@pytest.mark.parametrize("split", [0, 32])
@pytest.mark.parametrize("softcap,window", [(0.0, 0), (30.0, 0), (0.0, 40)])
def test_paged_decode_matches_reference(Hq, Hkv, D, split, softcap, window):
    from rl_project_b200.ops import _ext

    C = _ext.native()
    torch.manual_seed(0)
    B, max_blocks, num_blocks = 5, 12, 80
    k_pool = torch.randn(num_blocks, Hkv, BLOCK, D, device="cuda").bfloat16()
    v_pool = torch.randn(num_blocks, Hkv, BLOCK, D, device="cuda").bfloat16()
    perm = torch.randperm(num_blocks)[: B * max_blocks].view(B, max_blocks)
    tables = perm.int().cuda()
    lens = torch.tensor([1, 17, 100, 191, 64], dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, D, device="cuda").bfloat16()
    scale = 1.0 / math.sqrt(D)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = C.paged_decode(q, k_pool, v_pool, tables, lens, split, scale, softcap, window, status)
    ref = _reference(q, k_pool, v_pool, tables, lens, scale, softcap, window)
    assert int(status.item()) == 0
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


def test_paged_write_scatters_rows():
    from rl_project_b200.ops import _ext

    C = _ext.native()
    num_blocks, Hkv, D, B = 10, 2, 64, 3
    k_pool = torch.zeros(num_blocks, Hkv, BLOCK, D, device="cuda", dtype=torch.bfloat16)
    v_pool = torch.zeros_like(k_pool)
    k_new = torch.randn(B, Hkv, D, device="cuda").bfloat16()
    v_new = torch.randn(B, Hkv, D, device="cuda").bfloat16()
    blk = torch.tensor([7, 0, 3], dtype=torch.int32, device="cuda")
    off = torch.tensor([5, 15, 0], dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.paged_write(k_new, v_new, k_pool, v_pool, blk, off, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for b in range(B):
        assert torch.equal(k_pool[blk[b], :, off[b]], k_new[b])
        assert torch.equal(v_pool[blk[b], :, off[b]], v_new[b])
    assert int((k_pool != 0).any(-1).sum()) == B * Hkv


def test_paged_decode_reports_bad_block_id():
    from rl_project_b200.ops import _ext

    C = _ext.native()
    k_pool = torch.randn(4, 1, BLOCK, 64, device="cuda").bfloat16()
    tables = torch.tensor([[0, 99]], dtype=torch.int32, device="cuda")  # 99 is out of range: skipped + reported
    lens = torch.tensor([20], dtype=torch.int32, device="cuda")
    q = torch.randn(1, 2, 64, device="cuda").bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = C.paged_decode(q, k_pool, k_pool, tables, lens, 0, 0.125, 0.0, 0, status)
    torch.cuda.synchronize()
    assert int(status.item()) != 0
    assert torch.isfinite(out.float()).all()
