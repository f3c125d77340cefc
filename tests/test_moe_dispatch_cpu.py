"""Host-side MoE layout and the atomic-free dispatch / combine, on CPU against direct formulations."""
import torch

from rl_project_b200.ops.grouped_gemm import ALIGN, grouped_layout, rows_bound
from rl_project_b200.ops.moe_dispatch import combine, dispatch, row_maps


def _route(N=37, E=6, k=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(N)])
    idx[:5] = torch.tensor([0, 1])  # crowd one expert pair
    return idx


def test_grouped_layout():
    idx = _route()
    flat = idx.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=6)
    lay = grouped_layout(flat[order], counts)
    assert lay.rows == rows_bound(flat.numel(), 6) and lay.rows % ALIGN == 0
    padded = (counts + ALIGN - 1) // ALIGN * ALIGN
    assert torch.equal(lay.seg_len.long(), padded)
    assert torch.equal(lay.seg_start.long(), torch.cumsum(padded, 0) - padded)
    # every slot lands inside its expert's segment, rows are distinct
    e_sorted = flat[order]
    assert torch.all(lay.dest >= lay.seg_start.long()[e_sorted])
    assert torch.all(lay.dest < (lay.seg_start + lay.seg_len).long()[e_sorted])
    assert lay.dest.unique().numel() == lay.dest.numel()
    for t, g in enumerate(lay.tile_group.tolist()):
        r0 = t * ALIGN
        if g < 0:
            assert r0 >= int(padded.sum())
        else:
            assert int(lay.seg_start[g]) <= r0 < int(lay.seg_start[g] + lay.seg_len[g])


def test_dispatch_combine_match_index_add_and_gradients():
    torch.manual_seed(0)
    N, E, k, C = 37, 6, 2, 5
    idx = _route(N, E, k)
    flat = idx.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=E)
    lay = grouped_layout(flat[order], counts)
    maps = row_maps(order, lay.dest, lay.rows, k)
    x = torch.randn(N, C, dtype=torch.float64, requires_grad=True)
    w = torch.rand(N, k, dtype=torch.float64, requires_grad=True)
    W = torch.randn(E, C, C, dtype=torch.float64)
    # the buffer path: dispatch, a per-row "expert" map, combine
    xp = dispatch(x, maps)
    e_of_row = torch.full((lay.rows,), -1)
    for e in range(E):
        e_of_row[int(lay.seg_start[e]):int(lay.seg_start[e] + counts[e])] = e
    y = torch.stack([xp[r] @ W[e] if e >= 0 else xp[r] * 0 for r, e in enumerate(e_of_row.tolist())])
    out = combine(y, w, maps)
    # the direct formulation: index_select / index_add over (token, slot)
    tok = order // k
    ys = torch.stack([x[t] @ W[e] for t, e in zip(tok.tolist(), flat[order].tolist())])
    ref = torch.zeros(N, C, dtype=torch.float64).index_add_(0, tok, ys * w.reshape(-1)[order, None])
    torch.testing.assert_close(out, ref)
    g = torch.randn(N, C, dtype=torch.float64)
    gx, gw = torch.autograd.grad(out, (x, w), g)
    rx, rw = torch.autograd.grad(ref, (x, w), g)
    torch.testing.assert_close(gx, rx)
    torch.testing.assert_close(gw, rw)
