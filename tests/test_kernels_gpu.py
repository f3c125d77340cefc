"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF = torch.bfloat16


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item() + 1e-6
    assert err <= tol * max(1.0, scale), f"max err {err} (scale {scale})"


def test_native_library_loaded():
    from rl_project_b200.ops._ext import available, native

    assert available()
    native()


@pytest.mark.parametrize("dim", [64, 512, 2048, 4096])
@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm(dim, residual):
    from rl_project_b200.ops.norm import add_rms_norm, rms_norm

    rows = 257
    x = torch.randn(rows, dim, device=DEV, dtype=BF, requires_grad=True)
    d = torch.randn(rows, dim, device=DEV, dtype=BF, requires_grad=True)
    w = (1 + 0.1 * torch.randn(dim, device=DEV)).to(BF).requires_grad_()
    gy = torch.randn(rows, dim, device=DEV, dtype=BF)
    gh = torch.randn(rows, dim, device=DEV, dtype=BF)
    xr, dr, wr = x.detach().float().requires_grad_(), d.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    if residual:
        h, y = add_rms_norm(x, d, w)
        (y.float() * gy.float()).sum().add_((h.float() * gh.float()).sum()).backward()
        hr = xr + dr
        yr = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
        ((yr * gy.float()).sum() + (hr * gh.float()).sum()).backward()
        _close(h, hr, 1e-2)
        _close(d.grad, dr.grad, 3e-2)
    else:
        y = rms_norm(x, w)
        (y.float() * gy.float()).sum().backward()
        yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
        (yr * gy.float()).sum().backward()
    _close(y, yr, 2e-2)
    _close(x.grad, xr.grad, 3e-2)
    _close(w.grad, wr.grad, 3e-2)


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 8, 2), (128, 4, 4)])
def test_rope_split(D, Hq, Hkv):
    from rl_project_b200.ops.rope import RopeTable, apply_rope_reference, rope_split_qkv

    B, T = 2, 33
    tab = RopeTable(D, theta=500000.0, max_seq_len=64)
    qkv = torch.randn(B, T, (Hq + 2 * Hkv) * D, device=DEV, dtype=BF, requires_grad=True)
    q, k, v = rope_split_qkv(qkv, tab, Hq, Hkv, D, offset=3)
    ref = qkv.detach().float().requires_grad_()
    rq, rk, rv = ref.split([Hq * D, Hkv * D, Hkv * D], -1)
    rq = rq.reshape(B, T, Hq, D).transpose(1, 2)
    rk = rk.reshape(B, T, Hkv, D).transpose(1, 2)
    rv = rv.reshape(B, T, Hkv, D).transpose(1, 2)
    cos, sin = tab.tables(64, torch.device(DEV))
    rq = apply_rope_reference(rq, cos[3:3 + T], sin[3:3 + T])
    rk = apply_rope_reference(rk, cos[3:3 + T], sin[3:3 + T])
    _close(q, rq, 1e-2)
    _close(k, rk, 1e-2)
    _close(v, rv, 1e-2)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    ((q.float() * gq.float()).sum() + (k.float() * gk.float()).sum() + (v.float() * gv.float()).sum()).backward()
    ((rq * gq.float()).sum() + (rk * gk.float()).sum() + (rv * gv.float()).sum()).backward()
    _close(qkv.grad, ref.grad, 2e-2)


def test_swiglu():
    from rl_project_b200.ops.activation import swiglu

    h = torch.randn(300, 2 * 1024, device=DEV, dtype=BF, requires_grad=True)
    hr = h.detach().float().requires_grad_()
    y = swiglu(h)
    g, u = hr.chunk(2, -1)
    yr = F.silu(g) * u
    _close(y, yr, 2e-2)
    gy = torch.randn_like(y)
    (y.float() * gy.float()).sum().backward()
    (yr * gy.float()).sum().backward()
    _close(h.grad, hr.grad, 3e-2)


@pytest.mark.parametrize("V", [256, 50257, 128256])
def test_logprob_kernel(V):
    from rl_project_b200.ops._ext import native

    N = 64
    logits = (3 * torch.randn(N, V, device=DEV)).to(BF)
    tgt = torch.randint(0, V, (N,), device=DEV)
    tgt[::7] = -1
    lse, lp, ent = native().logprob_fwd(logits, tgt, True, None)
    lf = logits.float()
    ref_logp = torch.log_softmax(lf, -1)
    ref_lp = ref_logp.gather(1, tgt.clamp(min=0)[:, None]).squeeze(1) * (tgt >= 0)
    ref_ent = -(ref_logp.exp() * ref_logp).sum(-1)
    _close(lse, torch.logsumexp(lf, -1), 1e-4)
    _close(lp, ref_lp, 1e-4)
    _close(ent, ref_ent, 1e-3)
    g_lp = torch.randn(N, device=DEV)
    g_ent = torch.randn(N, device=DEV)
    lg = logits.clone()
    native().logprob_bwd_(lg, tgt, lse, g_lp, ent, g_ent, 1.0)
    lr = lf.clone().requires_grad_()
    lpr = torch.log_softmax(lr, -1)
    lpt = lpr.gather(1, tgt.clamp(min=0)[:, None]).squeeze(1) * (tgt >= 0)
    er = -(lpr.exp() * lpr).sum(-1)
    ((lpt * g_lp).sum() + (er * g_ent).sum()).backward()
    _close(lg, lr.grad, 2e-2)


def test_linear_logprobs_grads():
    from rl_project_b200.ops.logprob import linear_cross_entropy

    N, d, V = 512, 256, 3000
    h = (0.5 * torch.randn(N, d, device=DEV)).to(BF).requires_grad_()
    W = (0.05 * torch.randn(V, d, device=DEV)).to(BF).requires_grad_()
    t = torch.randint(0, V, (N,), device=DEV)
    t[:100] = -1
    loss = linear_cross_entropy(h, W, t)
    loss.backward()
    hr, Wr = h.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    lr = F.cross_entropy(hr @ Wr.t(), t, ignore_index=-1)
    lr.backward()
    assert abs(loss.item() - lr.item()) < 2e-2
    _close(h.grad, hr.grad, 5e-2)
    _close(W.grad, Wr.grad, 5e-2)


def test_embedding():
    from rl_project_b200.ops.embedding import embedding

    V, D = 1000, 256
    W = torch.randn(V, D, device=DEV, dtype=BF, requires_grad=True)
    idx = torch.randint(0, V, (4, 300), device=DEV)
    idx[0, :50] = 7  # many repeats of one id
    y = embedding(idx, W)
    _close(y, W.detach()[idx], 0)
    gy = torch.randn_like(y)
    y.backward(gy)
    ref = torch.zeros(V, D, device=DEV).index_add_(0, idx.reshape(-1), gy.reshape(-1, D).float())
    _close(W.grad, ref, 2e-2)


def test_fused_adamw_matches_torch():
    from rl_project_b200.ops.optim import FusedAdamW

    torch.manual_seed(1)
    shapes = [(300, 200), (200,), (70000,)]
    masters = [torch.randn(s, device=DEV) for s in shapes]
    p16 = [torch.nn.Parameter(m.to(BF)) for m in masters]
    p32 = [torch.nn.Parameter(m.to(BF).float()) for m in masters]  # masters start from the bf16 weights
    opt = FusedAdamW([{"params": p16[:1] + p16[2:], "weight_decay": 0.1}, {"params": p16[1:2], "weight_decay": 0.0}],
                     lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    ref = torch.optim.AdamW([{"params": p32[:1] + p32[2:], "weight_decay": 0.1},
                             {"params": p32[1:2], "weight_decay": 0.0}], lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    for _ in range(5):
        grads = [torch.randn(s, device=DEV) for s in shapes]
        for p, g in zip(p16, grads):
            p.grad = g.to(BF)
        for p, g in zip(p32, grads):
            p.grad = g.to(BF).float()
        norm = opt.clip_grad_norm(1.0)
        ref_norm = torch.nn.utils.clip_grad_norm_(p32, 1.0)
        assert abs(norm.item() - ref_norm.item()) < 1e-3 * ref_norm.item()
        opt.step()
        ref.step()
    for p, q in zip(p16, p32):
        _close(opt.state[p]["master"], q.detach(), 1e-4)
        _close(p, q.detach(), 1e-2)


def test_nf4_dequant_matches_cpu():
    from rl_project_b200.models.quantization.nf4 import dequantize_nf4, quantize_nf4

    w = torch.randn(96, 130)
    packed, absmax, shape = quantize_nf4(w)
    cpu = dequantize_nf4(packed, absmax, shape)
    gpu = dequantize_nf4(packed.cuda(), absmax.cuda(), shape, torch.bfloat16)
    _close(gpu.cpu(), cpu, 1e-2)


def test_model_step_on_gpu_decreases_loss():
    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.ops.optim import FusedAdamW

    spec = model_spec_from_preset("bl_tiny", block_size=128, n_embd=128, n_head=4, n_kv_head=2, d_ff=256)
    m = TransformerLM(spec).cuda().to(BF)
    opt = FusedAdamW(m.parameters(), lr=3e-3)
    x = torch.randint(0, 256, (4, 128), device=DEV)
    losses = []
    for _ in range(20):
        opt.zero_grad()
        _, loss = m(x, x)
        loss.backward()
        opt.clip_grad_norm(1.0)
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 0.5, losses


def test_model_matches_fp32_reference_forward():
    """bf16 GPU path (fused kernels) vs the same weights on the fp32 CPU path."""
    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.transformer.model import TransformerLM

    spec = model_spec_from_preset("bl_tiny", block_size=128, n_embd=128, n_head=4, n_kv_head=2, d_ff=256)
    cpu = TransformerLM(spec)
    gpu = TransformerLM(spec)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.cuda().to(BF)
    x = torch.randint(0, 256, (2, 128))
    _, l_cpu = cpu(x, x)
    _, l_gpu = gpu(x.cuda(), x.cuda())
    assert abs(l_cpu.item() - l_gpu.item()) < 2e-2 * max(1.0, l_cpu.item())


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (300, 200, 136), (1024, 3072, 2048)])
def test_tcgen05_gemm_all_layouts(M, N, K):
    from rl_project_b200.ops.gemm import gemm_nn, gemm_nt, gemm_tn

    a = torch.randn(M, K, device=DEV).to(BF)
    b = torch.randn(N, K, device=DEV).to(BF)
    ref = a.float() @ b.float().t()
    _close(gemm_nt(a, b), ref, 1e-2)
    # dgrad form: a [M, K] @ c [K, N]
    c = torch.randn(K, N, device=DEV).to(BF)
    _close(gemm_nn(a, c), a.float() @ c.float(), 1e-2)
    # wgrad form: a[K', M]^T @ d[K', N]
    d = torch.randn(M, N, device=DEV).to(BF)
    e = torch.randn(M, K, device=DEV).to(BF)
    _close(gemm_tn(d, e), d.float().t() @ e.float(), 1e-2)
    acc = torch.ones(N, K, device=DEV)
    gemm_tn(d, e, out=acc, accumulate=True)
    _close(acc, d.float().t() @ e.float() + 1, 1e-2)


def test_tcgen05_linear_autograd():
    from rl_project_b200.ops import gemm

    x = torch.randn(4, 96, 512, device=DEV).to(BF).requires_grad_()
    w = (0.05 * torch.randn(768, 512, device=DEV)).to(BF).requires_grad_()
    y = gemm._Linear.apply(x.reshape(-1, 512), w)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = xr.reshape(-1, 512) @ wr.t()
    yr.backward(gy.float())
    _close(y, yr, 1e-2)
    _close(x.grad, xr.grad, 2e-2)
    _close(w.grad, wr.grad, 2e-2)


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (300, 520, 192), (64, 256, 1024)])
def test_nf4_gemm_matches_dequantised_matmul(M, N, K):
    from rl_project_b200.models.quantization.nf4 import NF4_TABLE, dequantize_nf4, quantize_nf4
    from rl_project_b200.ops._ext import native

    g = torch.Generator().manual_seed(M + N)
    w = torch.randn(N, K, generator=g) * 0.05
    packed, absmax, shape = quantize_nf4(w)
    wd = dequantize_nf4(packed, absmax, shape).cuda()  # fp32 oracle of the quantised weight
    packed, absmax, table = packed.cuda(), absmax.float().cuda(), NF4_TABLE.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.randn(M, K, generator=g).cuda().bfloat16()
    dy = torch.randn(M, N, generator=g).cuda().bfloat16()
    y = native().nf4_gemm(x, packed, absmax, table, 0, N, K, status)
    dx = native().nf4_gemm(dy, packed, absmax, table, 1, N, K, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for got, ref in ((y, x.float() @ wd.t()), (dx, dy.float() @ wd)):
        rel = ((got.float() - ref).norm() / ref.norm()).item()
        assert rel < 1e-2, rel
