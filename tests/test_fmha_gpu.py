"""Own tcgen05 attention (csrc/fmha_fwd.cu, csrc/fmha_bwd.cu) against an fp32 PyTorch reference of the same
op: forward output and log-sum-exp, backward dq / dk / dv through autograd, the paired-head forward (even
GQA groups) and the one-head kernel (odd groups, MLA d_qk 192), causal / non-causal, sliding window, tanh
soft-cap, ragged and odd sequence lengths.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,Hq,Hkv,D,causal", [
    (1, 128, 1, 1, 128, True),
    (2, 256, 4, 2, 128, True),
    (1, 300, 2, 1, 64, True),      # ragged last tile (zero-filled rows past T)
    (2, 384, 8, 8, 64, False),
    (1, 1024, 4, 1, 128, True),
])
def test_fmha_forward_matches_fp32(B, T, Hq, Hkv, D, causal):
    from rl_project_b200.ops.attention import attention_reference, fmha_check, fmha_forward

    g = torch.Generator(device="cuda").manual_seed(T + D)
    # token-major storage, as the fused RoPE kernel writes it
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).bfloat16().transpose(1, 2)
    k = torch.randn(B, T, Hkv, D, device="cuda", generator=g).bfloat16().transpose(1, 2)
    v = torch.randn(B, T, Hkv, D, device="cuda", generator=g).bfloat16().transpose(1, 2)
    out, lse = fmha_forward(q, k, v, causal=causal, with_lse=True)
    torch.cuda.synchronize()
    fmha_check(q.device)
    ref = attention_reference(q.float(), k.float(), v.float(), causal=causal, q_offset=0).float()
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err
    rep = Hq // Hkv
    kk = k.float().repeat_interleave(rep, 1)
    s = (q.float() @ kk.transpose(-1, -2)) * D ** -0.5
    if causal:
        s = s.masked_fill(torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    assert (lse - torch.logsumexp(s, -1)).abs().max().item() < 1e-2


@pytest.mark.parametrize("B,T,Hq,Hkv,D,causal", [
    (1, 128, 1, 1, 128, True),
    (2, 256, 4, 2, 64, True),
    (1, 300, 2, 1, 128, True),
    (1, 256, 2, 2, 64, False),
    (1, 301, 4, 2, 64, True),      # T not a multiple of 4: the log-sum-exp rows are read element by element
    (2, 640, 8, 2, 128, True),     # several query tiles and heads per key tile (d 128: dQ drained in-step)
    (2, 640, 8, 2, 64, True),      # ... (d 64: dQ drained one step later, double-buffered tiles)
])
def test_fmha_backward_matches_fp32_autograd(B, T, Hq, Hkv, D, causal):
    from rl_project_b200.ops.attention import attention_reference, fmha, fmha_check

    g = torch.Generator(device="cuda").manual_seed(7 * T + D)
    mk = lambda h: torch.randn(B, T, h, D, device="cuda", generator=g).bfloat16().transpose(1, 2)  # noqa: E731
    q, k, v = mk(Hq), mk(Hkv), mk(Hkv)
    do = mk(Hq)
    qs, ks, vs = (x.detach().requires_grad_(True) for x in (q, k, v))
    out = fmha(qs, ks, vs, causal=causal)
    out.backward(do)
    torch.cuda.synchronize()
    fmha_check(q.device)
    q32, k32, v32 = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    ref = attention_reference(q32, k32, v32, causal=causal, q_offset=0)
    ref.backward(do.float())
    for name, a, r in (("dq", qs.grad, q32.grad), ("dk", ks.grad, k32.grad), ("dv", vs.grad, v32.grad)):
        rel = ((a.float() - r).norm() / r.norm()).item()
        assert rel < 2e-2, (name, rel)


@pytest.mark.parametrize("T,causal", [(256, True), (200, False)])
def test_fmha_forward_mla_shape(T, causal):
    """d_qk 192 (128 no-RoPE + 64 RoPE dims) with d_v 128: the prefill shape of multi-head latent attention."""
    from rl_project_b200.ops.attention import attention_reference, fmha_check, fmha_forward

    g = torch.Generator(device="cuda").manual_seed(T)
    B, H = 1, 4
    q = torch.randn(B, T, H, 192, device="cuda", generator=g).bfloat16().transpose(1, 2)
    k = torch.randn(B, T, H, 192, device="cuda", generator=g).bfloat16().transpose(1, 2)
    v = torch.randn(B, T, H, 128, device="cuda", generator=g).bfloat16().transpose(1, 2)
    out, _ = fmha_forward(q, k, v, causal=causal)
    torch.cuda.synchronize()
    fmha_check(q.device)
    ref = attention_reference(q.float(), k.float(), v.float(), causal=causal, q_offset=0).float()
    assert out.shape == (B, H, T, 128)
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("T,window,softcap,D", [
    (512, 128, 0.0, 64),     # window equal to a tile: one or two key tiles per query tile
    (700, 200, 0.0, 128),    # window not a tile multiple, ragged T
    (384, 0, 30.0, 64),      # tanh soft-cap only
    (640, 96, 20.0, 128),    # both
])
def test_fmha_window_softcap_forward_backward(T, window, softcap, D):
    """Sliding window and tanh soft-cap against the fp32 reference: output, then dq / dk / dv by autograd."""
    from rl_project_b200.ops.attention import attention_reference, fmha, fmha_check

    B, Hq, Hkv = 2, 4, 2
    g = torch.Generator(device="cuda").manual_seed(T + window)
    # scaled so that the cap matters (logits of several cap widths)
    mk = lambda h: (2.0 * torch.randn(B, T, h, D, device="cuda", generator=g)).bfloat16().transpose(1, 2)  # noqa: E731
    q, k, v = mk(Hq), mk(Hkv), mk(Hkv)
    do = mk(Hq)
    qs, ks, vs = (x.detach().requires_grad_(True) for x in (q, k, v))
    out = fmha(qs, ks, vs, True, None, window, softcap)
    out.backward(do)
    torch.cuda.synchronize()
    fmha_check(q.device)
    q32, k32, v32 = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    ref = attention_reference(q32, k32, v32, window=window, softcap=softcap, causal=True, q_offset=0)
    ref.backward(do.float())
    rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 1e-2, rel
    for name, a, r in (("dq", qs.grad, q32.grad), ("dk", ks.grad, k32.grad), ("dv", vs.grad, v32.grad)):
        rel = ((a.float() - r).norm() / r.norm()).item()
        assert rel < 2e-2, (name, rel)


def test_causal_attention_routes_window_to_own_kernel():
    """On CUDA a windowed call goes through the own kernel (no T x T fp32 matrix) and matches the reference."""
    from rl_project_b200.ops import attention as A

    B, H, T, D = 1, 2, 1024, 64
    q, k, v = (torch.randn(B, T, H, D, device="cuda").bfloat16().transpose(1, 2) for _ in range(3))
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    with torch.no_grad():
        out = A.causal_attention(q, k, v, window=256)
    torch.cuda.synchronize()
    A.fmha_check(q.device)
    # the eager reference would hold B*H*T*T fp32 scores (8 MiB here); the kernel needs only out + lse
    assert torch.cuda.max_memory_allocated() - base < B * H * T * T * 4 // 4
    ref = A.attention_reference(q.float(), k.float(), v.float(), window=256, q_offset=0)
    assert (out.float() - ref.float()).abs().max().item() < 2e-2
