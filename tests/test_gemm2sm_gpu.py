"""The 2-SM tcgen05 GEMM (csrc/gemm_2sm.cu) against a plain fp32 PyTorch product of the same operands.

Covers the three operand layouts a linear layer needs (x W^T, dy W, dy^T x), bf16 and fp32 outputs,
accumulation into fp32 (TMA reduce-add), ragged M / N / K (tiles that run past the matrix), a strided
output (ldc > N), alpha, and a grid capped below the device's cluster count (more tiles per pair).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _rel(got, ref):
    return ((got.float() - ref).norm() / ref.norm().clamp_min(1e-12)).item()


def _status():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 256), (300, 200, 136), (1000, 1048, 520),
                                   (4096, 3072, 2048)])
@pytest.mark.parametrize("layout", ["nt", "nn", "tn"])
@pytest.mark.parametrize("nsub", [1, 2])
def test_gemm2sm_matches_fp32(M, N, K, layout, nsub):
    from rl_project_b200.ops._ext import native

    if layout == "tn" and M % 8:
        pytest.skip("A stored [K][M] needs M a multiple of 8 (16-byte TMA row pitch)")
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    st = _status()
    if layout == "nt":    # A [M][K], B [N][K]
        a = torch.randn(M, K, device="cuda", generator=g).to(BF)
        b = torch.randn(N, K, device="cuda", generator=g).to(BF)
        ref = a.float() @ b.float().t()
        args = (0, 0, K, K)
    elif layout == "nn":  # A [M][K], B [K][N]
        a = torch.randn(M, K, device="cuda", generator=g).to(BF)
        b = torch.randn(K, N, device="cuda", generator=g).to(BF)
        ref = a.float() @ b.float()
        args = (0, 1, K, N)
    else:                 # A [K][M], B [K][N]
        a = torch.randn(K, M, device="cuda", generator=g).to(BF)
        b = torch.randn(K, N, device="cuda", generator=g).to(BF)
        ref = a.float().t() @ b.float()
        args = (1, 1, M, N)
    a_mn, b_mn, lda, ldb = args
    out = torch.empty(M, N, device="cuda", dtype=BF)
    native().gemm2(a, b, out, a_mn, b_mn, 0, M, N, K, lda, ldb, N, 1.0, st, 0, nsub)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(out, ref) < 8e-3
    if layout != "nn":
        # fp32 store, then accumulate the same product on top with alpha 0.5 (TMA reduce-add)
        out32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
        native().gemm2(a, b, out32, a_mn, b_mn, 1, M, N, K, lda, ldb, N, 1.0, st, 0, nsub)
        native().gemm2(a, b, out32, a_mn, b_mn, 2, M, N, K, lda, ldb, N, 0.5, st, 0, nsub)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert _rel(out32, 1.5 * ref) < 1e-4


@pytest.mark.parametrize("M,N,K", [(512, 768, 1024), (300, 200, 1160), (1024, 1048, 4160)])
@pytest.mark.parametrize("layout", ["nt", "tn"])
@pytest.mark.parametrize("splits,group_m", [(2, 0), (3, 1), (5, 32)])
def test_gemm2sm_split_k_accumulates(M, N, K, layout, splits, group_m):
    """K split into ranges that each reduce-add their partial product into a zeroed fp32 C (ragged K: the
    ranges differ in length), under several raster group heights."""
    from rl_project_b200.ops._ext import native

    if layout == "tn" and M % 8:
        pytest.skip("A stored [K][M] needs M a multiple of 8")
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + 5 * K + splits)
    if layout == "nt":
        a = torch.randn(M, K, device="cuda", generator=g).to(BF)
        b = torch.randn(N, K, device="cuda", generator=g).to(BF)
        ref, args = a.float() @ b.float().t(), (0, 0, K, K)
    else:
        a = torch.randn(K, M, device="cuda", generator=g).to(BF)
        b = torch.randn(K, N, device="cuda", generator=g).to(BF)
        ref, args = a.float().t() @ b.float(), (1, 1, M, N)
    a_mn, b_mn, lda, ldb = args
    for nsub in (1, 2):
        out = torch.zeros(M, N, device="cuda", dtype=torch.float32)
        st = _status()
        native().gemm2x(a, b, out, a_mn, b_mn, 2, M, N, K, lda, ldb, N, 1.0, st, 0, nsub, splits, group_m)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert _rel(out, ref) < 1e-4


def test_weight_gradient_wrapper_splits_k():
    """gemm_tn with a bf16 output on a q|k|v-like weight gradient (few tiles, long K) takes the split path
    and matches the fp32 product; the split count comes from the wave model."""
    from rl_project_b200.ops import gemm

    M, N, K = 3072, 2048, 32768
    assert gemm.k_splits(M, N, K, 1, torch.cuda.current_device()) > 1
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(K, M, device="cuda", generator=g).to(BF)
    b = torch.randn(K, N, device="cuda", generator=g).to(BF)
    got = gemm.gemm_tn(a, b)
    assert got.dtype == BF
    assert _rel(got, a.float().t() @ b.float()) < 8e-3


@pytest.mark.parametrize("nsub", [1, 2])
def test_gemm2sm_strided_output_and_small_grid(nsub):
    """C written into columns [0, N) of a wider buffer; the grid capped at 4 CTAs (2 pairs)."""
    from rl_project_b200.ops._ext import native

    M, N, K, ldc = 1536, 640, 384, 1024
    a = torch.randn(M, K, device="cuda").to(BF)
    b = torch.randn(N, K, device="cuda").to(BF)
    buf = torch.full((M, ldc), 3.0, device="cuda", dtype=BF)
    st = _status()
    native().gemm2(a, b, buf, 0, 0, 0, M, N, K, K, K, ldc, 2.0, st, 4, nsub)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(buf[:, :N], 2.0 * (a.float() @ b.float().t())) < 8e-3
    assert bool((buf[:, N:] == 3.0).all())  # nothing written past N


@pytest.mark.parametrize("nsub", [1, 2])
def test_gemm2sm_agrees_with_one_sm_kernel(nsub):
    """The two own kernels give the same product (fp32 accumulation, bf16 output) on the same operands."""
    from rl_project_b200.ops._ext import native

    for (M, N, K) in [(384, 512, 320), (2048, 2048, 1024)]:
        a = torch.randn(M, K, device="cuda").to(BF)
        b = torch.randn(N, K, device="cuda").to(BF)
        o1 = torch.empty(M, N, device="cuda", dtype=BF)
        o2 = torch.empty(M, N, device="cuda", dtype=BF)
        native().gemm(a, b, o1, 0, 0, 0, M, N, K, K, K, N, 1.0, None)
        native().gemm2(a, b, o2, 0, 0, 0, M, N, K, K, K, N, 1.0, None, 0, nsub)
        torch.cuda.synchronize()
        assert _rel(o2, o1.float()) < 4e-3


def test_tma_launchers_work_from_a_fresh_thread():
    """A thread that has made no CUDA runtime call (like autograd's backward workers) can launch the TMA
    kernels: the launchers bind the device's primary context before encoding tensor maps."""
    import threading

    from rl_project_b200.ops import gemm

    a = torch.randn(512, 256, device="cuda").to(BF)
    b = torch.randn(384, 256, device="cuda").to(BF)
    ref = a.float() @ b.float().t()
    out, err = {}, []

    def work():
        try:
            out["y"] = gemm.gemm_nt(a, b)
            torch.cuda.current_stream().synchronize()
        except Exception as e:  # noqa: BLE001 - reported below
            err.append(repr(e))

    t = threading.Thread(target=work)
    t.start()
    t.join(120)
    assert not err, err
    assert _rel(out["y"], ref) < 8e-3


@pytest.mark.parametrize("mode", ["tuned", "hybrid", "fwd_dgrad"])
def test_tuned_and_hybrid_modes_linear_match_fp32(mode):
    """``tuned`` (per-shape choice among the 2-SM kernel's tile shapes and cuBLAS), ``hybrid`` (own forward,
    cuBLAS gradients) and ``fwd_dgrad`` (own forward and input gradient, cuBLAS weight gradient) give the fp32
    product in every layout of a linear layer; ``tuned`` records a choice for each shape it timed."""
    from rl_project_b200.ops import gemm

    old, old_min = gemm._MODE, gemm._MIN_TILES
    gemm._MODE, gemm._MIN_TILES = mode, 0  # small test shapes still take the own kernel
    try:
        x = torch.randn(1024, 512, device="cuda").to(BF).requires_grad_()
        w = (0.05 * torch.randn(1536, 512, device="cuda")).to(BF).requires_grad_()
        for _ in range(2):  # first call times the candidates, second replays the choice
            x.grad = w.grad = None
            y = gemm.linear(x, w)
            gy = torch.randn_like(y)
            y.backward(gy)
        xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
        yr = xr @ wr.t()
        yr.backward(gy.float())
        assert _rel(y, yr) < 8e-3 and _rel(x.grad, xr.grad) < 1e-2 and _rel(w.grad, wr.grad) < 1e-2
        if mode == "tuned":
            picks = gemm.tuned_choices()
            assert {(k[0], k[1]) for k in picks} >= {(0, 0), (0, 1), (1, 1)}
            assert set(picks.values()) <= {"own1", "own2", "cublas"}
    finally:
        gemm._MODE, gemm._MIN_TILES = old, old_min


@pytest.mark.parametrize("M,H,K", [(1024, 512, 256), (1000, 1408, 520), (4096, 2816, 2048)])
def test_swiglu_epilogue_matches_fp32(M, H, K):
    """One GEMM over [W1; W3] whose epilogue writes the projection and silu(gate) * up: both against an fp32
    product (hidden widths that are not a multiple of the 256-unit tile included)."""
    from rl_project_b200.ops import gemm

    g = torch.Generator(device="cuda").manual_seed(M + H + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(BF)
    w13 = (torch.randn(2 * H, K, device="cuda", generator=g) / K ** 0.5).to(BF)
    h13, act = gemm.gemm_nt_swiglu(x, w13)
    torch.cuda.synchronize()
    ref = x.float() @ w13.float().t()
    assert _rel(h13, ref) < 8e-3
    ref_act = torch.nn.functional.silu(ref[:, :H]) * ref[:, H:]
    assert _rel(act, ref_act) < 1.5e-2
    # the activation is computed from the stored bf16 projection, as the standalone kernel does
    from rl_project_b200.ops._ext import native

    assert _rel(act, native().swiglu_fwd(h13).float()) < 1e-3


def test_linear_swiglu_gradients_match_fp32():
    """Forward and both gradients of the fused projection + activation against fp32 autograd."""
    from rl_project_b200.ops import gemm

    old, old_min = gemm._MODE, gemm._MIN_TILES
    gemm._MODE, gemm._MIN_TILES = "tcgen05", 0
    try:
        M, H, K = 2048, 1024, 768
        x = torch.randn(M, K, device="cuda").to(BF).requires_grad_()
        w13 = (torch.randn(2 * H, K, device="cuda") / K ** 0.5).to(BF).requires_grad_()
        a = gemm.linear_swiglu(x, w13)
        da = torch.randn_like(a)
        a.backward(da)
        xr, wr = x.detach().float().requires_grad_(), w13.detach().float().requires_grad_()
        hr = xr @ wr.t()
        ar = torch.nn.functional.silu(hr[:, :H]) * hr[:, H:]
        ar.backward(da.float())
        assert _rel(a, ar) < 1.5e-2 and _rel(x.grad, xr.grad) < 2e-2 and _rel(w13.grad, wr.grad) < 2e-2
    finally:
        gemm._MODE, gemm._MIN_TILES = old, old_min


@pytest.mark.parametrize("M,N,K", [(600, 1000, 256), (4096, 32000, 512), (2048, 128256, 2048)])
def test_lse_epilogue_matches_logprob_pass(M, N, K):
    """LM-head forward whose epilogue writes per-chunk row statistics: the merged log-sum-exp, target log-prob
    and entropy equal the standalone pass over the same bf16 logits (ragged last tile included)."""
    from rl_project_b200.ops import gemm
    from rl_project_b200.ops._ext import native

    g = torch.Generator(device="cuda").manual_seed(M + N)
    h = torch.randn(M, K, device="cuda", generator=g).to(BF)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5 * 3).to(BF)
    tgt = torch.randint(0, N, (M,), device="cuda", generator=g)
    tgt[::7] = -1
    logits, stats = gemm.gemm_nt_lse(h, w)
    lse, lp, ent = native().logprob_combine(stats, logits, tgt, True, None)
    rlse, rlp, rent = native().logprob_fwd(logits, tgt, True, None)
    torch.cuda.synchronize()
    assert _rel(logits, h.float() @ w.float().t()) < 8e-3
    assert torch.allclose(lse, rlse, rtol=1e-5, atol=1e-4)
    assert torch.allclose(lp, rlp, rtol=1e-5, atol=1e-4)
    assert torch.allclose(ent, rent, rtol=1e-4, atol=1e-3)


def test_linear_logprobs_with_lse_epilogue_matches_fp32():
    """The fused-loss entry point takes the statistics epilogue when the own GEMM runs the LM head; log-probs
    and both gradients match an fp32 log-softmax."""
    from rl_project_b200.ops import gemm
    from rl_project_b200.ops.logprob import linear_logprobs, linear_logprobs_reference

    old, old_min, old_rows = gemm._MODE, gemm._MIN_TILES, gemm._LSE_MIN_ROWS
    gemm._MODE, gemm._MIN_TILES, gemm._LSE_MIN_ROWS = "hybrid", 0, 0
    try:
        M, V, K = 1024, 8192, 512
        h = torch.randn(M, K, device="cuda").to(BF).requires_grad_()
        w = (torch.randn(V, K, device="cuda") / K ** 0.5).to(BF).requires_grad_()
        tgt = torch.randint(0, V, (M,), device="cuda")
        assert gemm.lse_fusable(h.detach(), w.detach())
        lp, ent = linear_logprobs(h, w, tgt, with_entropy=True)
        (lp.sum() + 0.1 * ent.sum()).backward()
        hr, wr = h.detach().float().requires_grad_(), w.detach().float().requires_grad_()
        rlp, rent = linear_logprobs_reference(hr, wr, tgt, with_entropy=True)
        (rlp.sum() + 0.1 * rent.sum()).backward()
        assert (lp - rlp).abs().max().item() < 0.1 and _rel(ent, rent) < 1e-2
        assert _rel(h.grad, hr.grad) < 3e-2 and _rel(w.grad, wr.grad) < 3e-2
    finally:
        gemm._MODE, gemm._MIN_TILES, gemm._LSE_MIN_ROWS = old, old_min, old_rows


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 64), (16, 4, 128)])
def test_rope_qkv_epilogue_matches_unfused(Hq, Hkv, D):
    """One GEMM with RoPE and the q / k / v split in its epilogue against the projection followed by the RoPE
    kernel: forward outputs and the gradients of x and w."""
    from rl_project_b200.ops import gemm
    from rl_project_b200.ops.rope import RopeTable, rope_split_qkv

    old, old_min = gemm._MODE, gemm._MIN_TILES
    gemm._MODE, gemm._MIN_TILES = "hybrid", 0
    try:
        B, T, C = 2, 1024, 1024
        g = torch.Generator(device="cuda").manual_seed(D)
        x = torch.randn(B, T, C, device="cuda", generator=g).to(BF).requires_grad_()
        w = (torch.randn((Hq + 2 * Hkv) * D, C, device="cuda", generator=g) / C ** 0.5).to(BF).requires_grad_()
        table = RopeTable(D, 500000.0, max_seq_len=T)
        cos, sin = table.tables(T + 3, x.device)
        assert gemm.rope_qkv_fusable(x.detach().reshape(-1, C), w.detach(), Hq, Hkv, D)
        q, k, v = gemm.linear_rope_qkv(x, w, cos, sin, None, Hq, Hkv, D, offset=3)
        gq, gk, gv = (torch.randn_like(t) for t in (q, k, v))
        (q.float() * gq).sum().add_((k.float() * gk).sum()).add_((v.float() * gv).sum()).backward()
        dx, dw = x.grad.clone(), w.grad.clone()
        x.grad = w.grad = None
        qkv = (x.reshape(-1, C) @ w.t()).view(B, T, -1)
        rq, rk, rv = rope_split_qkv(qkv, table, Hq, Hkv, D, offset=3, heads_major=False)
        (rq.float() * gq).sum().add_((rk.float() * gk).sum()).add_((rv.float() * gv).sum()).backward()
        torch.cuda.synchronize()
        for got, ref in ((q, rq), (k, rk), (v, rv)):
            assert got.shape == ref.shape
            assert _rel(got, ref.float()) < 1e-2
        assert _rel(dx, x.grad.float()) < 1e-2 and _rel(dw, w.grad.float()) < 1e-2
    finally:
        gemm._MODE, gemm._MIN_TILES = old, old_min


@pytest.mark.parametrize("M,H,K", [(1000, 1408, 512), (4096, 2816, 2048)])
def test_dgrad_swiglu_epilogue_matches_unfused(M, H, K):
    """The down projection's input gradient with the SwiGLU backward in the epilogue equals dy W2 rounded to
    bf16 followed by the standalone activation backward."""
    from rl_project_b200.ops import gemm
    from rl_project_b200.ops._ext import native

    g = torch.Generator(device="cuda").manual_seed(M + H)
    dy = torch.randn(M, K, device="cuda", generator=g).to(BF)
    w2 = (torch.randn(K, H, device="cuda", generator=g) / H ** 0.5).to(BF)
    h13 = torch.randn(M, 2 * H, device="cuda", generator=g).to(BF)
    got = gemm.gemm_dgrad_swiglu(dy, w2, h13)
    ref = native().swiglu_bwd(h13, (dy.float() @ w2.float()).to(BF))
    torch.cuda.synchronize()
    assert _rel(got, ref.float()) < 1e-2


@pytest.mark.parametrize("fused_bwd", [False, True])
def test_swiglu_ffn_matches_fp32(fused_bwd):
    """Whole gated FFN on the fused epilogues (with and without the activation backward in the down projection's
    input-gradient GEMM): output and the gradients of x, [W1; W3] and W2 against fp32."""
    from rl_project_b200.ops import gemm

    old, old_min, old_bwd = gemm._MODE, gemm._MIN_TILES, gemm._SWIGLU_BWD
    gemm._MODE, gemm._MIN_TILES, gemm._SWIGLU_BWD = "hybrid", 0, fused_bwd
    try:
        M, C, H = 2048, 768, 2048
        x = torch.randn(M, C, device="cuda").to(BF).requires_grad_()
        w13 = (torch.randn(2 * H, C, device="cuda") / C ** 0.5).to(BF).requires_grad_()
        w2 = (torch.randn(C, H, device="cuda") / H ** 0.5).to(BF).requires_grad_()
        out = gemm.swiglu_ffn(x, w13, w2)
        gout = torch.randn_like(out)
        out.backward(gout)
        xr, w13r, w2r = (t.detach().float().requires_grad_() for t in (x, w13, w2))
        hr = xr @ w13r.t()
        outr = (torch.nn.functional.silu(hr[:, :H]) * hr[:, H:]) @ w2r.t()
        outr.backward(gout.float())
        assert _rel(out, outr) < 2e-2
        assert _rel(x.grad, xr.grad) < 3e-2 and _rel(w13.grad, w13r.grad) < 3e-2 and _rel(w2.grad, w2r.grad) < 3e-2
    finally:
        gemm._MODE, gemm._MIN_TILES, gemm._SWIGLU_BWD = old, old_min, old_bwd
