"""Model variants (GQA / MHA / MLA / NSA / MoE / MTP / windows / caps / RoPE scaling) on the CPU path."""

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.models.generation.sampling import apply_sampling_filters, generate_tokens
from rl_project_b200.models.transformer.model import TransformerLM

VARIANTS = [
    {},
    {"n_kv_head": 1},
    {"use_rope": False},
    {"use_swiglu": False},
    {"sliding_window": 8},
    {"sliding_window": 8, "alternating_layers": True, "attn_logit_cap": 30.0},
    {"rope_scaling_type": "linear", "rope_scaling_factor": 2.0},
    {"rope_scaling_type": "yarn", "rope_scaling_factor": 4.0},
    {"use_mla": True, "kv_lora_rank": 16, "qk_nope_head_dim": 16, "qk_rope_head_dim": 8, "v_head_dim": 16},
    {"use_mla": True, "kv_lora_rank": 16, "q_lora_rank": 24, "qk_nope_head_dim": 16, "qk_rope_head_dim": 8,
     "v_head_dim": 16},
    {"use_nsa": True, "nsa_block_size": 4, "nsa_top_k": 4, "nsa_window_size": 8},
    {"use_moe": True, "n_experts": 4, "n_experts_active": 2, "n_shared_experts": 1},
    {"use_moe": True, "n_experts": 8, "n_experts_active": 2, "score_func": "sigmoid", "aux_loss_free": True,
     "n_expert_groups": 4, "n_limited_groups": 2, "n_dense_layers": 1, "moe_d_ff": 32},
    {"n_predict_tokens": 3},
    {"d_ff": 96, "rope_theta": 500000.0, "tie_embeddings": False},
]


@pytest.mark.parametrize("over", VARIANTS, ids=[str(sorted(v)) for v in VARIANTS])
def test_forward_backward_generate(over):
    spec = model_spec_from_preset("tiny", vocab_size=50, block_size=32, **over)
    m = TransformerLM(spec)
    x = torch.randint(0, 50, (2, 24))
    _, loss = m(x, x)
    loss.backward()
    assert torch.isfinite(loss)
    assert all(p.grad is not None for n, p in m.named_parameters() if p.requires_grad and "mtp" not in n
               and "gate.weight" not in n and "compress" not in n) or spec.use_moe or spec.use_nsa
    m.eval()
    out = m.generate(x[:, :5], 4, temperature=0.0, use_cache=not spec.use_nsa)
    assert out.shape == (2, 9)


@pytest.mark.parametrize("over", [{}, {"n_kv_head": 1}, {"sliding_window": 6},
                                  {"use_mla": True, "kv_lora_rank": 16, "qk_nope_head_dim": 16, "qk_rope_head_dim": 8,
                                   "v_head_dim": 16}])
def test_cached_equals_uncached_greedy(over):
    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=40, block_size=48, **over)).eval()
    x = torch.randint(0, 40, (2, 7))
    a = generate_tokens(m, x, 10, temperature=0.0, use_cache=True)
    b = generate_tokens(m, x, 10, temperature=0.0, use_cache=False)
    assert torch.equal(a, b)


def test_state_dict_keys_match_reference_tree():
    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=40, use_moe=True, n_experts=2, n_shared_experts=1,
                                             n_predict_tokens=2))
    keys = set(m.state_dict())
    for k in ("transformer.wte.weight", "transformer.h.0.ln_1.weight", "transformer.h.0.attn.q_proj.weight",
              "transformer.h.0.attn.c_proj.weight", "transformer.h.0.ffn.gate.weight",
              "transformer.h.0.ffn.experts.1.w2.weight", "transformer.h.0.ffn.shared_experts.w3.weight",
              "transformer.ln_f.weight", "lm_head.weight", "mtp_modules.0.proj.weight"):
        assert k in keys, k


def test_sampling_filters():
    logits = torch.tensor([[1.0, 2.0, 3.0, 4.0]])
    f = apply_sampling_filters(logits, temperature=1.0, top_k=2)
    assert torch.isinf(f[0, :2]).all() and torch.isfinite(f[0, 2:]).all()
    f = apply_sampling_filters(logits, temperature=1.0, top_p=0.5)
    assert torch.isfinite(f[0, 3]) and torch.isinf(f[0, 0])
    f = apply_sampling_filters(logits, temperature=1.0, min_p=0.5)
    assert torch.isinf(f[0, 0]) and torch.isfinite(f[0, 3])
    f = apply_sampling_filters(logits, repetition_penalty=2.0, past_tokens=[3])
    assert f[0, 3] == 2.0


def test_moe_sort_dispatch_matches_mask_loop():
    from rl_project_b200.models.moe.layer import MoELayer

    spec = model_spec_from_preset("tiny", vocab_size=40, use_moe=True, n_experts=4, n_experts_active=2)
    layer = MoELayer(spec).eval()
    x = torch.randn(2, 5, spec.n_embd)
    y = layer(x)
    xf = x.reshape(-1, spec.n_embd)
    w, idx = layer.gate(xf)
    ref = torch.zeros_like(xf)
    for k in range(2):
        for e in range(4):
            sel = idx[:, k] == e
            if sel.any():
                ref[sel] += w[sel, k:k + 1] * layer.experts[e](xf[sel])
    assert torch.allclose(y.reshape(-1, spec.n_embd), ref, atol=1e-5)


def test_fmha_wrapper_shapes_and_layout():
    """Host-side checks of the tcgen05 attention wrapper (the kernels themselves need a GPU)."""
    from rl_project_b200.core.errors import KernelError
    from rl_project_b200.ops.attention import FMHA_SHAPES, _token_major, fmha_forward

    assert (128, 128) in FMHA_SHAPES and (192, 128) in FMHA_SHAPES and (96, 96) not in FMHA_SHAPES
    x = torch.randn(2, 5, 3, 8)                 # token-major storage [B, T, H, D]
    v = x.transpose(1, 2)                        # the [B, H, T, D] view attention receives
    assert _token_major(v).data_ptr() == x.data_ptr()  # no copy for token-major views
    heads_major = torch.randn(2, 3, 5, 8)
    assert _token_major(heads_major).is_contiguous() and torch.equal(_token_major(heads_major),
                                                                     heads_major.transpose(1, 2))
    q = torch.zeros(1, 2, 4, 96, dtype=torch.bfloat16)
    with pytest.raises(KernelError):
        fmha_forward(q, q, q)
    with pytest.raises(KernelError):  # 3 query heads do not group over 2 key/value heads
        fmha_forward(torch.zeros(1, 3, 4, 64, dtype=torch.bfloat16), torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16),
                     torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16))


def test_rope_table_stays_on_the_host_under_a_default_device():
    """Tables built while a non-CPU default device is active (a model constructed under ``torch.device``)
    are host tensors, so growing them later cannot mix devices."""
    from rl_project_b200.ops.rope import RopeTable

    with torch.device("meta"):
        table = RopeTable(64, max_seq_len=16)
    assert table.inv_freq.device.type == "cpu" and table._cos.device.type == "cpu"
    cos, sin = table.tables(64, torch.device("cpu"))  # grows the table outside the context
    assert cos.shape == (64, 32) and torch.isfinite(sin).all()


def test_nsa_shared_score_fine_branches_equal_per_branch_oracle():
    """The fused selected + window branches equal computing each branch on its own (gathered top-k values,
    separate window scores), combined with the same gates."""
    import torch.nn.functional as F

    from rl_project_b200.models.attention.sparse import NativeSparseAttention

    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=40, block_size=32, use_nsa=True, nsa_block_size=4,
                                  nsa_top_k=3, nsa_window_size=5)
    attn = NativeSparseAttention(spec).eval()
    x = torch.randn(2, 11, spec.n_embd)
    got, _ = attn(x)
    B, T, C = x.shape
    H, D = attn.n_head, attn.head_dim
    heads = lambda t: t.view(B, T, H, D).transpose(1, 2)  # noqa: E731
    q, k, v = heads(attn.q_proj(x)), heads(attn.k_proj(x)), heads(attn.v_proj(x))
    from rl_project_b200.ops.rope import apply_rope

    q, k = apply_rope(q, attn.rope), apply_rope(k, attn.rope)
    s = (q @ k.transpose(-2, -1)) * attn.scale
    causal = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    top_s, top_i = s.masked_fill(causal, float("-inf")).topk(3, dim=-1)
    vs = torch.gather(v.unsqueeze(2).expand(-1, -1, T, -1, -1), 3, top_i.unsqueeze(-1).expand(-1, -1, -1, -1, D))
    sel = (torch.softmax(top_s, -1).unsqueeze(-2) @ vs).squeeze(-2)
    qp, kp = torch.arange(T)[:, None], torch.arange(T)[None, :]
    win = torch.softmax(s.masked_fill(~((kp <= qp) & (qp - kp < 5)), float("-inf")), -1) @ v
    g = F.softmax(attn.gate(x).view(B, T, 3, H), dim=2).permute(0, 3, 1, 2)
    y = g[..., 0:1] * attn._compressed(q, k, v) + g[..., 1:2] * sel + g[..., 2:3] * win
    ref = attn.c_proj(y.transpose(1, 2).reshape(B, T, C))
    assert torch.allclose(got, ref, atol=1e-5), (got - ref).abs().max()
