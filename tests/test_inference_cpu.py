"""Inference engine, paged allocator and scheduler on CPU (paged path through the
PyTorch reference of the decode kernel)."""
from __future__ import annotations

import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.core.errors import ServingError
from rl_project_b200.inference import (GenerationRequest, InferenceEngine, OutOfBlocksError, PagedBlockAllocator,
                                       RequestStatus,
                                       SamplingParams, Scheduler)
from rl_project_b200.models.transformer.model import TransformerLM


def _model(**overrides):
    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=97, **overrides)
    return TransformerLM(spec).eval()


def _greedy_reference(model, prompt, n):
    idx = torch.tensor([prompt])
    out = model.generate(idx, n, temperature=0.0, use_cache=False)
    return out[0, len(prompt):].tolist()


GREEDY = SamplingParams(max_tokens=12, temperature=0.0, top_k=None)


def test_engine_greedy_matches_uncached_model_mixed_lengths():
    model = _model()
    eng = InferenceEngine(model, max_batch=4)
    prompts = [[5, 6, 7], list(range(1, 20)), [9], list(range(30, 47)), [3, 3, 3, 3, 3]]
    reqs = eng.generate_batch(prompts, GREEDY)
    for p, r in zip(prompts, reqs):
        assert r.status == RequestStatus.FINISHED and r.finish_reason == "length"
        assert r.generated_tokens == _greedy_reference(model, p, 12), p
    assert eng.paged and eng.allocator.used_blocks == 0
    st = eng.stats()
    assert st["completed"] == 5 and st["running"] == 0


def test_engine_window_and_softcap_layers():
    model = _model(sliding_window=8, alternating_layers=True, attn_logit_cap=20.0)
    eng = InferenceEngine(model, max_batch=3)
    prompts = [list(range(2, 25)), [4, 8], list(range(10, 21))]
    reqs = eng.generate_batch(prompts, GREEDY)
    for p, r in zip(prompts, reqs):
        assert r.generated_tokens == _greedy_reference(model, p, 12)


def test_prefix_sharing_and_copy_on_write():
    model = _model()
    eng = InferenceEngine(model, max_batch=8)
    prompt = list(range(1, 21))  # 20 tokens: the second block is partly filled and shared
    reqs = [eng.submit(prompt, GREEDY) for _ in range(4)]
    eng.step()
    assert eng.shared_prefills == 3
    eng.run_until_idle()
    ref = _greedy_reference(model, prompt, 12)
    for r in reqs:
        assert r.generated_tokens == ref
    assert eng.allocator.cow_copies >= 3
    assert eng.allocator.used_blocks == 0 and all(c == 0 for c in eng.allocator.refs)


def test_sampled_requests_and_stop_tokens():
    model = _model()
    eng = InferenceEngine(model, max_batch=4, eos_token_id=None)
    ref = _greedy_reference(model, [1, 2, 3], 12)
    stop = ref[4]
    r_stop = eng.submit([1, 2, 3], SamplingParams(max_tokens=12, temperature=0.0, stop_token_ids=[stop]))
    torch.manual_seed(1)
    r_samp = eng.submit([7, 8], SamplingParams(max_tokens=6, temperature=1.0, top_k=5, top_p=0.9))
    r_pen = eng.submit([7, 8, 9], SamplingParams(max_tokens=5, temperature=0.0, repetition_penalty=1.3))
    eng.run_until_idle()
    assert r_stop.finish_reason == "stop" and r_stop.generated_tokens[-1] == stop
    assert r_stop.generated_tokens == ref[: ref.index(stop) + 1]
    assert len(r_samp.generated_tokens) == 6 and all(0 <= t < 97 for t in r_samp.generated_tokens)
    assert len(r_pen.generated_tokens) == 5


def test_cancel_rejection_and_streaming():
    model = _model()
    eng = InferenceEngine(model, max_batch=1, max_seq_len=32)
    too_long = eng.submit(list(range(30)), SamplingParams(max_tokens=10, temperature=0.0))
    a = eng.submit([1, 2], SamplingParams(max_tokens=20, temperature=0.0))
    b = eng.submit([3, 4], SamplingParams(max_tokens=3, temperature=0.0))
    eng.step()
    assert too_long.status == RequestStatus.FAILED
    assert eng.cancel(a.id)
    eng.run_until_idle()
    assert a.status == RequestStatus.CANCELLED
    assert b.status == RequestStatus.FINISHED
    assert list(b.stream_tokens(timeout=1)) == b.generated_tokens
    with pytest.raises(ServingError):
        eng.submit([], GREEDY)


def test_background_loop():
    model = _model()
    eng = InferenceEngine(model, max_batch=2)
    eng.start()
    try:
        r = eng.submit([5, 6, 7], SamplingParams(max_tokens=4, temperature=0.0))
        toks = list(r.stream_tokens(timeout=30))
    finally:
        eng.stop()
    assert toks == _greedy_reference(model, [5, 6, 7], 4)


def test_contiguous_fallback_for_mla():
    model = _model(use_mla=True, kv_lora_rank=16, qk_rope_head_dim=8, qk_nope_head_dim=16, v_head_dim=16)
    eng = InferenceEngine(model, max_batch=3)
    assert not eng.paged
    prompts = [[1, 2, 3], [4, 5, 6], [7, 8]]
    reqs = eng.generate_batch(prompts, SamplingParams(max_tokens=5, temperature=0.0))
    for p, r in zip(prompts, reqs):
        assert r.generated_tokens == _greedy_reference(model, p, 5)


def test_allocator_refcounts_and_out_of_blocks():
    a = PagedBlockAllocator(block_size=4, max_blocks=5)
    a.allocate("x", 6)  # 2 blocks
    assert a.tables["x"] == [0, 1]
    a.allocate("y", 1)
    a.share_prefix("x", "y", 6)  # y drops its own block and shares x's two
    assert a.refs[:2] == [2, 2] and a.used_blocks == 2
    src_dst = a.append_token("y")  # position 6 lies in shared block 1 -> copy
    assert src_dst is not None and src_dst[0] == 1 and a.tables["y"][1] == src_dst[1]
    assert a.append_token("x") is None  # block 1 now owned by x alone
    a.free("x")
    assert a.refs[0] == 1  # still held by y
    a.free("y")
    assert a.used_blocks == 0
    a.allocate("z", 20)
    with pytest.raises(OutOfBlocksError):
        a.append_token("z")
    s = Scheduler(PagedBlockAllocator(block_size=4, max_blocks=2), max_batch=4, max_seq_len=64)
    assert s.stats()["pending"] == 0


def test_rollouts_through_paged_engine_match_generate():
    from rl_project_b200.models.policy import NativePolicy
    from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine

    model = _model()
    from rl_project_b200.data.tokenizers import CharTokenizer

    policy = NativePolicy(model, CharTokenizer.ascii())
    prompts = [torch.tensor([1, 2, 3]), torch.tensor([4, 5, 6]), torch.tensor([7, 8, 9, 10, 11])]
    outs = {}
    for backend in ("paged", "generate"):
        cfg = RolloutConfig(group_size=2, max_new_tokens=6, temperature=0.0, engine=backend, stop_token_ids=(13,))
        outs[backend] = RolloutEngine(policy, cfg).rollout_many(prompts)
    for ga, gb in zip(outs["paged"], outs["generate"]):
        for a, b in zip(ga, gb):
            assert a.response_ids.tolist() == b.response_ids.tolist()
            torch.testing.assert_close(a.old_logprobs, b.old_logprobs)


def test_graph_decode_staging_layout():
    """The host staging of a CUDA-graph decode step (checked on the host; the graphs themselves need CUDA)."""
    import numpy as np

    from rl_project_b200.inference.engine import InferenceEngine

    assert [InferenceEngine._pow2(n, 64) for n in (1, 2, 3, 5, 64, 70)] == [1, 2, 4, 8, 64, 70]
    Bb, Wb, pad, bs = 4, 4, 99, 16
    hv = np.full(5 * Bb + Bb * Wb, -7, dtype=np.int32)
    InferenceEngine.stage_graph_inputs(hv, [11, 12], [5, 17], [[3], [4, 8]], Bb, Wb, pad, bs)
    tok, pos, ctx, sblk, soff = (hv[i * Bb:(i + 1) * Bb].tolist() for i in range(5))
    tables = hv[5 * Bb:].reshape(Bb, Wb).tolist()
    assert tok == [11, 12, 0, 0] and pos == [5, 17, 0, 0] and ctx == [6, 18, 1, 1]
    assert sblk == [3, 8, pad, pad]  # block holding each new token: position // 16 of the table
    assert soff == [5, 1, 0, 0]
    assert tables == [[3, 0, 0, 0], [4, 8, 0, 0], [pad, 0, 0, 0], [pad, 0, 0, 0]]


def test_scheduler_fifo_budget_rejection_and_cancel():
    from rl_project_b200.core.errors import ServingError

    alloc = PagedBlockAllocator(block_size=4, max_blocks=64)
    s = Scheduler(alloc, max_batch=8, max_seq_len=64, prefill_token_budget=10)
    mk = lambda n, mt=4: GenerationRequest(prompt_tokens=list(range(1, n + 1)), params=SamplingParams(max_tokens=mt))  # noqa: E731
    a, b, too_long, c, d = mk(6), mk(6), mk(8, mt=100), mk(3), mk(2)
    for r in (a, b, too_long, c, d):
        s.submit(r)
    first = s.admit()  # budget 10: a (6) fits, b would make 12 -> next step
    assert [r.id for r in first] == [a.id] and a.status == RequestStatus.RUNNING
    second = s.admit()  # b (6); the over-long request fails at the head; c (3) -> 9; d would make 11
    assert [r.id for r in second] == [b.id, c.id]
    assert too_long.status == RequestStatus.FAILED and "max_seq_len" in too_long.error
    assert s.cancel(d.id) and d.status == RequestStatus.CANCELLED and not s.admit()
    assert s.cancel(b.id) and b.meta["cancel"] and not s.cancel("nope")
    s.retire(a, "stop")
    assert a.status == RequestStatus.FINISHED and list(a.stream_tokens(timeout=1)) == []
    with pytest.raises(ServingError):
        a.start()  # a terminal request never runs again
    st = s.stats()
    assert st["running"] == 2 and st["pending"] == 0 and st["completed"] == 1 and st["rejected"] == 1


def test_request_stream_reads_backlog_in_batches():
    r = GenerationRequest(prompt_tokens=[1])
    r.start()
    for t in (5, 6, 7):
        r.push_token(t)
    toks, done = r.read_tokens(0, timeout=0)
    assert toks == [5, 6, 7] and not done
    r.finish("length")
    assert r.read_tokens(3, timeout=0) == ([], True)
    assert list(r.stream_tokens(timeout=1)) == [5, 6, 7]
