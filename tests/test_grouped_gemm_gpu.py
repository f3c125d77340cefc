"""Grouped tcgen05 GEMMs (MoE experts) against an fp32 PyTorch reference, and the
MoE layer's grouped path against its per-expert loop."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layout(counts):
    from rl_project_b200.ops.grouped_gemm import grouped_layout

    ct = torch.tensor(counts, device="cuda")
    se = torch.repeat_interleave(torch.arange(len(counts), device="cuda"), ct)
    return grouped_layout(se, ct)


def _pad(x, lay):
    return x.new_zeros(lay.rows, x.shape[1]).index_copy(0, lay.dest, x)


def _segments(counts):
    out, s = [], 0
    for c in counts:
        out.append((s, s + c))
        s += c
    return out


COUNTS = [300, 0, 128, 1, 517, 64]


@pytest.mark.parametrize("N,K", [(256, 128), (384, 192), (200, 64)])
def test_grouped_nt_and_tn(N, K):
    from rl_project_b200.ops.grouped_gemm import grouped_nt, grouped_tn

    torch.manual_seed(0)
    E, S = len(COUNTS), sum(COUNTS)
    lay = _layout(COUNTS)
    x = torch.randn(S, K, device="cuda").bfloat16()
    w = (torch.randn(E, N, K, device="cuda") / K ** 0.5).bfloat16()
    y = grouped_nt(_pad(x, lay), w, lay.tile_group).index_select(0, lay.dest)
    dy = torch.randn(S, N, device="cuda").bfloat16()
    dw = grouped_tn(_pad(dy, lay), _pad(x, lay), lay.seg_start, lay.seg_len)
    for e, (a, b) in enumerate(_segments(COUNTS)):
        ref = x[a:b].float() @ w[e].float().t()
        torch.testing.assert_close(y[a:b].float(), ref, atol=3e-2, rtol=2e-2)
        refw = dy[a:b].float().t() @ x[a:b].float()
        torch.testing.assert_close(dw[e].float(), refw, atol=5e-2 * max(1, (b - a) ** 0.5), rtol=2e-2)


def test_grouped_nn():
    from rl_project_b200.ops.grouped_gemm import grouped_nn

    torch.manual_seed(1)
    E, S, N, K = len(COUNTS), sum(COUNTS), 256, 192
    lay = _layout(COUNTS)
    dy = torch.randn(S, N, device="cuda").bfloat16()
    w = (torch.randn(E, N, K, device="cuda") / N ** 0.5).bfloat16()
    dx = grouped_nn(_pad(dy, lay), w, lay.tile_group).index_select(0, lay.dest)
    for e, (a, b) in enumerate(_segments(COUNTS)):
        torch.testing.assert_close(dx[a:b].float(), dy[a:b].float() @ w[e].float(), atol=3e-2, rtol=2e-2)


def test_moe_experts_grouped_matches_loop():
    import copy

    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.moe.layer import MoELayer

    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=97, use_moe=True, n_experts=8, n_experts_active=2,
                                  n_embd=128, moe_d_ff=192, n_shared_experts=1)
    lay = MoELayer(spec).cuda().bfloat16()
    ref = copy.deepcopy(lay).float()  # same (bf16-valued) weights, fp32 per-expert loop
    counts = [50, 0, 130, 7, 64, 200, 1, 12]
    xs = torch.randn(sum(counts), 128, device="cuda").bfloat16().requires_grad_(True)
    xr = xs.detach().float().requires_grad_(True)
    assert lay._grouped_ready(xs) and not ref._grouped_ready(xr)
    yb = lay.run_experts(xs, counts)
    yr = ref.run_experts(xr, counts)
    torch.testing.assert_close(yb.float(), yr, atol=3e-2, rtol=3e-2)
    g = torch.randn_like(yr)
    yb.backward(g.bfloat16())
    yr.backward(g)
    torch.testing.assert_close(xs.grad.float(), xr.grad, atol=5e-2, rtol=5e-2)
    for (n, pb), (_, pr) in zip(lay.experts.named_parameters(), ref.experts.named_parameters()):
        if pr.grad is None or pr.grad.abs().max() == 0:
            assert pb.grad is None or pb.grad.abs().max() == 0, n
            continue
        torch.testing.assert_close(pb.grad.float(), pr.grad, atol=8e-2, rtol=5e-2, msg=n)
    # the packed buffers hold the parameters: a second pass reuses them without copying
    w13 = lay._pack["w13"]
    lay.run_experts(xs, counts)
    assert lay._pack["w13"] is w13


def test_moe_layer_grouped_matches_loop(monkeypatch):
    """The whole layer (router, dispatch, grouped experts, combine) against the per-expert loop on the same
    bf16 layer, so both paths route identically."""
    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.moe.layer import MoELayer

    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=97, use_moe=True, n_experts=8, n_experts_active=2,
                                  n_embd=128, moe_d_ff=192, n_shared_experts=1)
    lay = MoELayer(spec).cuda().bfloat16()
    x = torch.randn(4, 96, 128, device="cuda").bfloat16()
    g = torch.randn(4, 96, 128, device="cuda").bfloat16()
    outs = {}
    for mode in ("1", "0", "1"):  # grouped, loop, grouped again (gradients accumulate into the packed sink)
        monkeypatch.setenv("RLB_MOE_GROUPED", mode)
        lay.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(True)
        y = lay(xi)
        y.backward(g)
        outs.setdefault(mode, []).append((y.detach().float(), xi.grad.float(),
                                          {n: p.grad.float().clone() for n, p in lay.named_parameters()
                                           if p.grad is not None}))
    (yg, dxg, pg), (yl, dxl, pl) = outs["1"][0], outs["0"][0]
    torch.testing.assert_close(yg, yl, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(dxg, dxl, atol=3e-2, rtol=3e-2)
    assert set(pg) == set(pl) or set(pl) <= set(pg)
    for n in pl:
        torch.testing.assert_close(pg[n], pl[n], atol=5e-2, rtol=5e-2, msg=n)
    y2, dx2, p2 = outs["1"][1]
    torch.testing.assert_close(y2, yg, atol=0, rtol=0)
    for n in pg:
        torch.testing.assert_close(p2[n], pg[n], atol=1e-2, rtol=1e-2, msg=n)
