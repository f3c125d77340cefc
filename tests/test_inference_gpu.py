"""Inference engine on the GPU: paged decode kernels inside the full model."""
from __future__ import annotations

import pytest
import torch

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.inference import InferenceEngine, SamplingParams
from rl_project_b200.models.transformer.model import TransformerLM

pytestmark = pytest.mark.gpu


def _model(n_embd, n_head, n_kv_head, **kw):
    torch.manual_seed(0)
    spec = ModelSpec(n_layer=2, n_head=n_head, n_kv_head=n_kv_head, n_embd=n_embd, block_size=512, dropout=0.0,
                     vocab_size=512, **kw)
    return TransformerLM(spec).cuda().bfloat16().eval()


def _check_greedy(model, prompt, generated, tol=0.08):
    """Every generated token is (up to bf16 rounding) the argmax of the full forward."""
    ids = torch.tensor([prompt + generated], device="cuda")
    with torch.no_grad():
        logits = model.full_logits(ids)[0].float()
    P = len(prompt)
    for i, tok in enumerate(generated):
        row = logits[P - 1 + i]
        assert row[tok] >= row.max() - tol, (i, tok, int(row.argmax()), float(row.max() - row[tok]))


@pytest.mark.parametrize("n_embd,n_head,n_kv,extra", [
    (256, 4, 1, {}),                                              # head_dim 64, 4 q heads per kv head
    (512, 4, 2, {}),                                              # head_dim 128, GQA 2
    (256, 4, 2, {"sliding_window": 24, "alternating_layers": True, "attn_logit_cap": 30.0}),
])
def test_engine_greedy_matches_full_forward(n_embd, n_head, n_kv, extra):
    model = _model(n_embd, n_head, n_kv, **extra)
    eng = InferenceEngine(model, max_batch=6)
    assert eng.paged
    prompts = [[1, 2, 3], list(range(5, 305)), [7], list(range(40, 57)), list(range(100, 180)), [9] * 33]
    reqs = eng.generate_batch(prompts, SamplingParams(max_tokens=16, temperature=0.0, top_k=None))
    for p, r in zip(prompts, reqs):
        assert len(r.generated_tokens) == 16
        _check_greedy(model, p, r.generated_tokens)
    assert eng.allocator.used_blocks == (1 if eng.decode_graphs else 0)  # graph decode keeps a padding block


def test_engine_prefix_sharing_gpu():
    model = _model(256, 4, 1)
    eng = InferenceEngine(model, max_batch=8)
    prompt = list(range(3, 40))
    greedy = SamplingParams(max_tokens=10, temperature=0.0, top_k=None)
    reqs = [eng.submit(prompt, greedy) for _ in range(4)]
    sampled = [eng.submit(prompt, SamplingParams(max_tokens=10, temperature=1.0, top_k=20)) for _ in range(4)]
    eng.run_until_idle()
    assert eng.shared_prefills == 7
    for r in reqs[1:]:
        assert r.generated_tokens == reqs[0].generated_tokens
    _check_greedy(model, prompt, reqs[0].generated_tokens)
    for r in sampled:
        assert len(r.generated_tokens) == 10 and all(0 <= t < 512 for t in r.generated_tokens)
    assert eng.allocator.used_blocks == (1 if eng.decode_graphs else 0)  # graph decode keeps a padding block


def test_graph_decode_matches_eager_decode():
    """The same greedy requests decoded eagerly and from captured graphs give the same tokens, across
    batch sizes that hit several (batch, width) buckets and with padding rows in play."""
    model = _model(512, 4, 2)
    prompts = [[1, 2, 3], list(range(5, 205)), [7], list(range(40, 57)), list(range(100, 180))]
    outs = {}
    for graphs in (False, True):
        eng = InferenceEngine(model, max_batch=8, decode_graphs=graphs)
        reqs = eng.generate_batch(prompts, SamplingParams(max_tokens=24, temperature=0.0, top_k=None))
        outs[graphs] = [r.generated_tokens for r in reqs]
        if graphs:
            assert eng._graphs, "no decode graph was captured"
            assert eng.allocator.used_blocks == 1  # only the padding block stays reserved
    assert outs[True] == outs[False]
