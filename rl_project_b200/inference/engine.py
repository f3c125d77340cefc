"""Continuous-batching inference engine over a paged KV cache.

Behaviour of ``src/forgeline/inference/engine.py:45-190`` (submit / step /
run_until_idle / generate / background loop / stats; per-request sampling
params; stop tokens, ``max_tokens``, cancellation and ``max_seq_len`` retire a
request and free its blocks at once so waiting requests join mid-flight),
built differently:

* every running sequence decodes in ONE batched step per engine step, whatever
  its length: K/V live in a device block pool and the decode kernel gathers
  each sequence's blocks through its block table (the reference groups
  sequences by equal length and concatenates / splits per-sequence caches);
* prompts of equal length admitted together are prefilled as one batch;
* a request whose prompt equals that of a running sequence shares its prompt
  blocks (copy-on-write on the first partly filled block) and reuses its
  prefill logits instead of running the prompt again -- the G samples of one
  GRPO prompt cost one prefill;
* the step's addressing (tokens, positions, slots, block tables) goes to the
  device as one pinned int32 copy, and the sampled tokens come back in one
  read.

Models whose attention is not grouped-query (MLA, NSA) decode through the
model's own contiguous ``step`` cache, grouped by length as in the reference.
"""

from __future__ import annotations

import threading
import time
from collections import defaultdict
from typing import Any, Dict, List, Optional, Tuple

import torch

from rl_project_b200.core.errors import ServingError
from rl_project_b200.inference.paged_memory import KERNEL_BLOCK, OutOfBlocksError, PagedBlockAllocator, PagedKVCache
from rl_project_b200.inference.requests import GenerationRequest, SamplingParams
from rl_project_b200.inference.scheduler import Scheduler
from rl_project_b200.models.generation.sampling import apply_sampling_filters, sample_from_logits
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.observability.tracing import Tracer

log = get_logger("forgeline.inference")


class _Seq:
    __slots__ = ("req", "position", "last_logits", "tokens", "cache")

    def __init__(self, req: GenerationRequest):
        self.req = req
        self.position = 0  # tokens whose K/V are cached
        self.last_logits: Optional[torch.Tensor] = None  # [1, V] logits of the prompt's last token
        self.tokens: List[int] = list(req.prompt_tokens)
        self.cache: Optional[List[Any]] = None  # contiguous per-layer cache (non-paged models only)


class InferenceEngine:
    def __init__(self, model: Any, *, max_batch: int = 8, max_seq_len: Optional[int] = None, block_size: int = 16,
                 max_blocks: Optional[int] = None, device: Optional[torch.device] = None,
                 eos_token_id: Optional[int] = None, share_prefixes: bool = True):
        self.model = model.eval()
        self.device = device or next(model.parameters()).device
        self.max_seq_len = min(max_seq_len or model.spec.block_size, model.spec.block_size)
        max_blocks = max_blocks or max_batch * ((self.max_seq_len + block_size - 1) // block_size + 1)
        self.paged = bool(getattr(model, "supports_paged_decode", lambda: False)())
        if self.paged and block_size != KERNEL_BLOCK:
            raise ServingError(f"paged decoding uses {KERNEL_BLOCK}-token blocks (got block_size={block_size})")
        self.allocator = PagedBlockAllocator(block_size=block_size, max_blocks=max_blocks)
        self.scheduler = Scheduler(self.allocator, max_batch=max_batch, max_seq_len=self.max_seq_len)
        self.kv: Optional[PagedKVCache] = None
        if self.paged:
            n_layer, n_kv, hd = model.kv_layout()
            dtype = next(model.parameters()).dtype
            self.kv = PagedKVCache(n_layer, n_kv, hd, max_blocks, self.device, dtype=dtype)
        self.eos_token_id = eos_token_id
        self.share_prefixes = share_prefixes and self.paged
        self.states: Dict[str, _Seq] = {}
        self._prefix_owner: Dict[Tuple[int, ...], str] = {}
        self._prompt_logits: Dict[str, torch.Tensor] = {}  # prompt-end logits, reused by prefix sharers
        self._sms = (torch.cuda.get_device_properties(self.device).multi_processor_count
                     if self.device.type == "cuda" else 0)
        self.tracer = Tracer()
        self.total_tokens = 0
        self.prefill_tokens = 0
        self.shared_prefills = 0
        self.decode_steps = 0
        self._pinned: Optional[torch.Tensor] = None
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self._lock = threading.Lock()

    # ------------------------------------------------------------ submission
    def submit(self, prompt_tokens: List[int], params: Optional[SamplingParams] = None,
               **kwargs: Any) -> GenerationRequest:
        params = params or SamplingParams()
        params.validate()
        if not prompt_tokens:
            raise ServingError("prompt must contain at least one token")
        req = GenerationRequest(prompt_tokens=list(prompt_tokens), params=params, **kwargs)
        self.scheduler.submit(req)
        return req

    def cancel(self, request_id: str) -> bool:
        return self.scheduler.cancel(request_id)

    # ------------------------------------------------------------ one engine step
    @torch.no_grad()
    def step(self) -> int:
        """Admit + prefill new requests, then decode one token for every running one."""
        with self._lock:
            produced = 0
            admitted = self.scheduler.admit()
            if admitted:
                produced += self._prefill(admitted)
            running = [s for s in self.states.values() if not s.req.finished and s.position > 0
                       and s.last_logits is None]
            if running:
                produced += self._decode(running) if self.paged else self._decode_contiguous(running)
            self.total_tokens += produced
            return produced

    # ------------------------------------------------------------ prefill
    def _prefill(self, reqs: List[GenerationRequest]) -> int:
        fresh: Dict[int, List[_Seq]] = defaultdict(list)
        shared: List[Tuple[_Seq, _Seq]] = []
        for req in reqs:
            st = _Seq(req)
            self.states[req.id] = st
            req.started_at = time.time()
            key = tuple(req.prompt_tokens)
            owner = self.states.get(self._prefix_owner.get(key, "")) if self.share_prefixes else None
            if owner is not None and owner.req.id != req.id:
                shared.append((st, owner))
            else:
                if self.share_prefixes:
                    self._prefix_owner[key] = req.id
                fresh[len(req.prompt_tokens)].append(st)
        produced = 0
        for T, group in fresh.items():
            try:
                with self.tracer.span("prefill", tokens=T * len(group), batch=len(group)):
                    self._prefill_group(group, T)
                self.prefill_tokens += T * len(group)
            except Exception as exc:  # noqa: BLE001
                for st in group:
                    self._fail(st, exc)
        for st, owner in shared:
            if owner.req.id not in self.states or self.states[owner.req.id] is not owner:
                # the prompt's owner retired in this step before its copy was taken: prefill normally
                try:
                    self._prefill_group([st], len(st.req.prompt_tokens))
                except Exception as exc:  # noqa: BLE001
                    self._fail(st, exc)
                continue
            self.allocator.share_prefix(owner.req.id, st.req.id, len(st.req.prompt_tokens))
            st.position = len(st.req.prompt_tokens)
            st.last_logits = self._prompt_logits[owner.req.id]
            self.shared_prefills += 1
        # first token of every newly admitted sequence, from its prompt logits
        new = [st for st in (s for g in fresh.values() for s in g) if st.req.id in self.states]
        new += [st for st, _ in shared if st.req.id in self.states and st.last_logits is not None]
        if new:
            produced += self._sample_and_emit(new, torch.cat([st.last_logits for st in new], 0))
            for st in new:
                st.last_logits = None
        return produced

    def _prefill_group(self, group: List[_Seq], T: int) -> None:
        ids = torch.tensor([st.req.prompt_tokens for st in group], dtype=torch.long).to(self.device,
                                                                                         non_blocking=True)
        logits, cache = self.model.prefill(ids)
        logits = logits.float()
        for i, st in enumerate(group):
            st.position = T
            st.last_logits = logits[i:i + 1]
            self._prompt_logits[st.req.id] = st.last_logits
            if self.paged:
                table = self.allocator.tables[st.req.id]
                for layer, (k, v) in enumerate(cache):
                    self.kv.write_prefix(layer, k[i], v[i], table)
            else:
                st.cache = [tuple(t[i:i + 1] for t in c) if isinstance(c, tuple) else c[i:i + 1] for c in cache]

    # ------------------------------------------------------------ decode
    def _decode(self, seqs: List[_Seq]) -> int:
        B = len(seqs)
        bs = self.allocator.block_size
        width = max(len(self.allocator.tables[s.req.id]) for s in seqs)
        n = 5 * B + B * width
        if self._pinned is None or self._pinned.numel() < n:
            self._pinned = torch.empty(max(n, 1024), dtype=torch.int32,
                                       pin_memory=self.device.type == "cuda")
        host = self._pinned[:n]
        hv = host.numpy()
        hv[:] = 0
        max_pos = 0
        max_ctx = 0
        for b, s in enumerate(seqs):
            table = self.allocator.tables[s.req.id]
            pos = s.position
            hv[b] = s.tokens[-1]
            hv[B + b] = pos
            hv[2 * B + b] = pos + 1
            hv[3 * B + b] = table[pos // bs]
            hv[4 * B + b] = pos % bs
            hv[5 * B + b * width: 5 * B + b * width + len(table)] = table
            max_pos = max(max_pos, pos)
            max_ctx = max(max_ctx, pos + 1)
        dev = host.to(self.device, non_blocking=True)
        from rl_project_b200.models.attention.causal import PagedDecodeMeta

        meta = PagedDecodeMeta(positions=dev[B:2 * B].view(B, 1), max_pos=max_pos, ctx_lens=dev[2 * B:3 * B],
                               slot_block=dev[3 * B:4 * B], slot_off=dev[4 * B:5 * B],
                               block_tables=dev[5 * B:].view(B, width),
                               split_tokens=self._split_tokens(B, max_ctx))
        try:
            with self.tracer.span("decode", batch=B):
                logits = self.model.decode_paged(dev[:B].long(), self.kv, meta).float()
        except Exception as exc:  # noqa: BLE001
            if self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()  # the pinned buffer is reused next step
            for s in seqs:
                self._fail(s, exc)
            return 0
        self.decode_steps += 1
        for s in seqs:
            s.position += 1
        return self._sample_and_emit(seqs, logits)

    def _split_tokens(self, B: int, max_ctx: int) -> int:
        """Split long contexts over several CTAs when the batch alone cannot fill the GPU."""
        if self.device.type != "cuda" or max_ctx <= 256:
            return 0
        ctas = B * self.model.spec.n_kv_head
        if ctas >= self._sms:
            return 0
        splits = min((2 * self._sms + ctas - 1) // ctas, max_ctx // 128)
        if splits <= 1:
            return 0
        per = (max_ctx + splits - 1) // splits
        return (per + KERNEL_BLOCK - 1) // KERNEL_BLOCK * KERNEL_BLOCK

    def _decode_contiguous(self, seqs: List[_Seq]) -> int:
        groups: Dict[int, List[_Seq]] = defaultdict(list)
        for s in seqs:
            groups[s.position].append(s)
        produced = 0
        for pos, group in groups.items():
            try:
                with self.tracer.span("decode", batch=len(group)):
                    nxt = torch.tensor([[s.tokens[-1]] for s in group], dtype=torch.long, device=self.device)
                    n_layers = len(group[0].cache)
                    merged = []
                    for i in range(n_layers):
                        parts = [s.cache[i] for s in group]
                        if isinstance(parts[0], tuple):
                            merged.append(tuple(torch.cat([p[j] for p in parts], 0) for j in range(len(parts[0]))))
                        else:
                            merged.append(torch.cat(parts, 0))
                    logits, new_cache = self.model.step(nxt, merged, pos)
            except Exception as exc:  # noqa: BLE001
                for s in group:
                    self._fail(s, exc)
                continue
            for b, s in enumerate(group):
                s.cache = [tuple(t[b:b + 1] for t in c) if isinstance(c, tuple) else c[b:b + 1] for c in new_cache]
                s.position += 1
            produced += self._sample_and_emit(group, logits.float())
        return produced

    # ------------------------------------------------------------ sampling
    def _sample_and_emit(self, seqs: List[_Seq], logits: torch.Tensor) -> int:
        B = len(seqs)
        out = torch.empty(B, dtype=torch.long, device=logits.device)
        groups: Dict[tuple, List[int]] = defaultdict(list)
        for i, s in enumerate(seqs):
            p = s.req.params
            if p.repetition_penalty != 1.0:
                f = apply_sampling_filters(logits[i:i + 1], p.temperature, p.top_k, p.top_p, p.min_p,
                                           p.repetition_penalty, s.tokens)
                out[i] = sample_from_logits(f, p.temperature).view(())
            else:
                groups[p.filter_key()].append(i)
        for (temp, top_k, top_p, min_p), rows in groups.items():
            idx = torch.as_tensor(rows, device=logits.device)
            sub = logits if len(rows) == B else logits.index_select(0, idx)
            if temp <= 0:
                tok = sub.argmax(-1)
            else:
                tok = sample_from_logits(apply_sampling_filters(sub, temp, top_k, top_p, min_p), temp).view(-1)
            if len(rows) == B:
                out = tok
            else:
                out.index_copy_(0, idx, tok)
        tokens = out.tolist()
        produced = 0
        for s, tok in zip(seqs, tokens):
            produced += self._emit(s, int(tok))
        return produced

    def _emit(self, st: _Seq, token: int) -> int:
        req, p = st.req, st.req.params
        req.push_token(token)
        st.tokens.append(token)
        stop = set(p.stop_token_ids)
        if self.eos_token_id is not None:
            stop.add(self.eos_token_id)
        if token in stop:
            self._retire(st, "stop")
        elif len(req.generated_tokens) >= p.max_tokens:
            self._retire(st, "length")
        elif req.meta.get("cancel"):
            self._retire(st, "cancelled")
        elif st.position + 1 >= self.max_seq_len:
            self._retire(st, "length")
        else:
            try:
                cow = self.allocator.append_token(req.id)
                if cow is not None and self.kv is not None:
                    self.kv.copy_block(*cow)
            except OutOfBlocksError as exc:
                self._fail(st, exc)
        return 1

    # ------------------------------------------------------------ retirement
    def _forget(self, st: _Seq) -> None:
        rid = st.req.id
        self.states.pop(rid, None)
        self._prompt_logits.pop(rid, None)
        key = tuple(st.req.prompt_tokens)
        if self._prefix_owner.get(key) == rid:
            del self._prefix_owner[key]
        st.cache = None

    def _retire(self, st: _Seq, reason: str) -> None:
        self._forget(st)
        self.scheduler.retire(st.req, reason)

    def _fail(self, st: _Seq, exc: BaseException) -> None:
        log.error("sequence_failed", request=st.req.id, error=repr(exc))
        self._forget(st)
        self.scheduler.retire(st.req, "error", error=f"{type(exc).__name__}: {exc}")

    # ------------------------------------------------------------ blocking helpers
    def run_until_idle(self, max_steps: int = 10_000) -> None:
        for _ in range(max_steps):
            if not self.scheduler.has_work():
                return
            self.step()
        raise ServingError("engine did not become idle within max_steps")

    def generate(self, prompt_tokens: List[int], params: Optional[SamplingParams] = None) -> GenerationRequest:
        req = self.submit(prompt_tokens, params)
        while not req.finished:
            self.step()
        return req

    def generate_batch(self, prompts: List[List[int]], params: Optional[SamplingParams] = None) -> List[GenerationRequest]:
        """Submit every prompt, run until all finish, return the requests in order."""
        reqs = [self.submit(p, params) for p in prompts]
        while not all(r.finished for r in reqs):
            self.step()
        return reqs

    # ------------------------------------------------------------ background loop (serving)
    def start(self, poll_interval: float = 0.005) -> None:
        if self._thread is not None:
            return
        self._stop.clear()

        def loop() -> None:
            while not self._stop.is_set():
                if self.scheduler.has_work():
                    self.step()
                else:
                    time.sleep(poll_interval)

        self._thread = threading.Thread(target=loop, daemon=True, name="forgeline-engine")
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5.0)
            self._thread = None

    def stats(self) -> Dict[str, Any]:
        out = {**self.scheduler.stats(), "total_tokens": self.total_tokens, "prefill_tokens": self.prefill_tokens,
               "shared_prefills": self.shared_prefills, "decode_steps": self.decode_steps, "paged": self.paged,
               "spans": self.tracer.summary()}
        if self.kv is not None:
            out["kv_cache_bytes"] = self.kv.nbytes
        return out
