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

On CUDA the paged decode step is replayed from CUDA graphs (default; ``decode_graphs=False`` or
``RLB_DECODE_GRAPHS=0`` launches it eagerly) instead of launching its ~10 kernels per layer from
the host: one graph per (batch, block-table width) bucket, both rounded up to a power of two,
captured on first use.  Padding rows decode a dummy token into a block reserved for them, so they
never touch a live sequence's K/V.  Graphs hold the model's weight and KV-pool addresses: call
``reset_graphs()`` after replacing (not updating in place) a weight tensor.  Measured on B200 with
the dense 1B model, batch 64: 26.9k generated tokens/s against 13.5k eager, identical greedy tokens.
"""

from __future__ import annotations

import os
import threading
import time
from collections import defaultdict
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from rl_project_b200.core.errors import ServingError
from rl_project_b200.inference.paged_memory import KERNEL_BLOCK, OutOfBlocksError, PagedBlockAllocator, PagedKVCache
from rl_project_b200.inference.requests import GenerationRequest, SamplingParams
from rl_project_b200.inference.scheduler import Scheduler
from rl_project_b200.models.generation.sampling import apply_sampling_filters, sample_from_logits
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.observability.tracing import Tracer
from rl_project_b200.ops.paged_attention import paged_write

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
                 eos_token_id: Optional[int] = None, share_prefixes: bool = True, profile: bool = False,
                 decode_graphs: Optional[bool] = None):
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
        self.profile = profile and self.device.type == "cuda"
        self._prof: Dict[str, float] = {}
        self._sample_calls = 0
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self._lock = threading.Lock()
        # CUDA-graph decode (paged models on CUDA only)
        if decode_graphs is None:
            decode_graphs = os.environ.get("RLB_DECODE_GRAPHS", "1") == "1"
        self.max_batch = max_batch
        self._graphs: Dict[Tuple[int, int], Any] = {}
        self._graph_pool: Any = None
        self._graph_fail: set = set()
        self._pad_block = -1
        self.decode_graphs = bool(decode_graphs) and self.paged and self.device.type == "cuda"
        if self.decode_graphs:
            self._pad_block = self.allocator.allocate("__graph_padding__", 1)[0]

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
    PREFILL_BUCKET = 64  # prompts are right-padded to a multiple of this and prefilled together
    PREFILL_TOKENS = 1 << 16  # tokens per prefill forward

    def _prefill(self, reqs: List[GenerationRequest]) -> int:
        fresh: List[_Seq] = []
        shared: List[Tuple[_Seq, _Seq]] = []
        vocab = int(self.model.spec.vocab_size)
        for req in reqs:
            st = _Seq(req)
            self.states[req.id] = st
            req.started_at = time.time()
            if min(req.prompt_tokens) < 0 or max(req.prompt_tokens) >= vocab:
                # fail this request alone, before its ids reach a batched forward with other requests
                self._fail(st, ServingError(f"prompt token id outside the vocabulary [0, {vocab})"))
                continue
            key = tuple(req.prompt_tokens)
            owner = self.states.get(self._prefix_owner.get(key, "")) if self.share_prefixes else None
            if owner is not None and owner.req.id != req.id:
                shared.append((st, owner))
            else:
                if self.share_prefixes:
                    self._prefix_owner[key] = req.id
                fresh.append(st)
        for group in self._prefill_batches(fresh):
            n_tok = sum(len(st.req.prompt_tokens) for st in group)
            try:
                with self.tracer.span("prefill", tokens=n_tok, batch=len(group)):
                    self._prefill_group(group)
                self.prefill_tokens += n_tok
            except Exception as exc:  # noqa: BLE001
                for st in group:
                    self._fail(st, exc)
        for st, owner in shared:
            if self.states.get(owner.req.id) is not owner or owner.req.id not in self._prompt_logits:
                # the prompt's owner failed in this step before its prefix could be shared: prefill normally
                try:
                    self._prefill_group([st])
                except Exception as exc:  # noqa: BLE001
                    self._fail(st, exc)
                continue
            self.allocator.share_prefix(owner.req.id, st.req.id, len(st.req.prompt_tokens))
            st.position = len(st.req.prompt_tokens)
            st.last_logits = self._prompt_logits[owner.req.id]
            self.shared_prefills += 1
        # first token of every newly admitted sequence, from its prompt logits
        new = [st for st in fresh if st.req.id in self.states and st.last_logits is not None]
        new += [st for st, _ in shared if st.req.id in self.states and st.last_logits is not None]
        produced = 0
        if new:
            produced += self._sample_and_emit(new, torch.cat([st.last_logits for st in new], 0))
            for st in new:
                st.last_logits = None
        return produced

    def _prefill_batches(self, seqs: List[_Seq]) -> List[List[_Seq]]:
        """Paged: prompts grouped by padded length (a multiple of PREFILL_BUCKET), at most PREFILL_TOKENS
        per forward.  Contiguous caches: grouped by exact length (no padding may enter the cache)."""
        q = self.PREFILL_BUCKET
        buckets: Dict[int, List[_Seq]] = defaultdict(list)
        for st in seqs:
            n = len(st.req.prompt_tokens)
            buckets[min(-(-n // q) * q, self.max_seq_len) if self.paged else n].append(st)
        out: List[List[_Seq]] = []
        for L, group in sorted(buckets.items()):
            per = max(1, self.PREFILL_TOKENS // max(L, 1))
            out.extend(group[i:i + per] for i in range(0, len(group), per))
        return out

    def _prefill_group(self, group: List[_Seq]) -> None:
        lens = [len(st.req.prompt_tokens) for st in group]
        L = max(lens)
        if self.paged:
            L = min(-(-L // self.PREFILL_BUCKET) * self.PREFILL_BUCKET, self.max_seq_len)
        rows = torch.zeros(len(group), L, dtype=torch.long)
        for i, st in enumerate(group):
            rows[i, :lens[i]] = torch.as_tensor(st.req.prompt_tokens, dtype=torch.long)
        ids = rows.to(self.device, non_blocking=True)
        last = torch.as_tensor([n - 1 for n in lens], dtype=torch.long)
        logits, cache = self.model.prefill(ids, last_positions=last)
        logits = logits.float()
        for i, st in enumerate(group):
            st.position = lens[i]
            st.last_logits = logits[i:i + 1]
            self._prompt_logits[st.req.id] = st.last_logits
            if not self.paged:
                st.cache = [tuple(t[i:i + 1] for t in c) if isinstance(c, tuple) else c[i:i + 1] for c in cache]
        if not self.paged:
            return
        # one gather and one slot write per layer for every prompt token of the batch
        bs = self.allocator.block_size
        flat, blocks, offs = [], [], []
        for i, st in enumerate(group):
            pos = torch.arange(lens[i])
            flat.append(pos + i * L)
            blocks.append(torch.as_tensor(self.allocator.tables[st.req.id], dtype=torch.int64)[pos // bs])
            offs.append(pos % bs)
        packed = torch.cat([torch.cat(flat), torch.cat(blocks), torch.cat(offs)]).to(self.device, non_blocking=True)
        n_tok = packed.numel() // 3
        flat_d = packed[:n_tok]
        blk_d, off_d = packed[n_tok:2 * n_tok].to(torch.int32), packed[2 * n_tok:].to(torch.int32)
        for layer, (k, v) in enumerate(cache):
            B, H, _, D = k.shape
            kk = k.transpose(1, 2).reshape(B * L, H, D).index_select(0, flat_d)
            vv = v.transpose(1, 2).reshape(B * L, H, D).index_select(0, flat_d)
            kl, vl = self.kv.layer(layer)
            paged_write(kk, vv, kl, vl, blk_d, off_d)

    # ------------------------------------------------------------ profiling (CUDA events per decode step)
    @staticmethod
    def _event():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def reset_profile(self) -> None:
        self._prof = {}

    def profile_summary(self) -> Dict[str, float]:
        n = max(1.0, self._prof.get("steps", 0.0))
        out = {k: v / n for k, v in self._prof.items() if k != "steps"}
        out["steps"] = self._prof.get("steps", 0.0)
        return out

    def _account(self, evs: List[Any], t_host0: float) -> None:
        torch.cuda.synchronize(self.device)
        p = self._prof
        p["forward_ms"] = p.get("forward_ms", 0.0) + evs[0].elapsed_time(evs[1])
        p["sampling_ms"] = p.get("sampling_ms", 0.0) + evs[2].elapsed_time(evs[3])
        p["step_wall_ms"] = p.get("step_wall_ms", 0.0) + (time.perf_counter() - t_host0) * 1e3
        p["steps"] = p.get("steps", 0.0) + 1

    # ------------------------------------------------------------ decode
    def _decode(self, seqs: List[_Seq]) -> int:
        if self.decode_graphs and not self.profile:
            try:
                done = self._decode_graph(seqs)
            except Exception as exc:  # noqa: BLE001
                torch.cuda.current_stream(self.device).synchronize()
                import traceback

                log.error("decode_graph_step_failed", error=repr(exc), where=traceback.format_exc(limit=6))
                for s in seqs:
                    self._fail(s, exc)
                return 0
            if done is not None:
                return done
        t_host0 = time.perf_counter()
        B = len(seqs)
        bs = self.allocator.block_size
        tables = [self.allocator.tables[s.req.id] for s in seqs]
        width = max(len(t) for t in tables)
        n = 5 * B + B * width
        if self._pinned is None or self._pinned.numel() < n:
            self._pinned = torch.empty(max(n, 1024), dtype=torch.int32,
                                       pin_memory=self.device.type == "cuda")
        host = self._pinned[:n]
        hv = host.numpy()
        pos = np.fromiter((s.position for s in seqs), dtype=np.int64, count=B)
        hv[:B] = np.fromiter((s.tokens[-1] for s in seqs), dtype=np.int64, count=B)
        hv[B:2 * B] = pos
        hv[2 * B:3 * B] = pos + 1
        hv[4 * B:5 * B] = pos % bs
        grid = hv[5 * B:].reshape(B, width)
        grid[:] = 0
        for b, t in enumerate(tables):
            grid[b, :len(t)] = t
        hv[3 * B:4 * B] = grid[np.arange(B), pos // bs]
        max_pos = int(pos.max())
        dev = host.to(self.device, non_blocking=True)
        from rl_project_b200.models.attention.causal import PagedDecodeMeta

        meta = PagedDecodeMeta(positions=dev[B:2 * B].view(B, 1), max_pos=max_pos, ctx_lens=dev[2 * B:3 * B],
                               slot_block=dev[3 * B:4 * B], slot_off=dev[4 * B:5 * B],
                               block_tables=dev[5 * B:].view(B, width),
                               split_tokens=self._split_tokens(B, max_pos + 1))
        evs = [self._event()] if self.profile else None
        try:
            with self.tracer.span("decode", batch=B):
                logits = self.model.decode_paged(dev[:B].long(), self.kv, meta)
        except Exception as exc:  # noqa: BLE001
            if self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()  # the pinned buffer is reused next step
            for s in seqs:
                self._fail(s, exc)
            return 0
        if evs is not None:
            evs.append(self._event())
        self.decode_steps += 1
        for s in seqs:
            s.position += 1
        produced = self._sample_and_emit(seqs, logits, evs)
        if evs is not None:
            self._account(evs, t_host0)
        return produced

    # ------------------------------------------------------------ CUDA-graph decode
    @staticmethod
    def _pow2(n: int, cap: int) -> int:
        b = 1
        while b < n:
            b *= 2
        return max(n, min(b, cap))

    @staticmethod
    def stage_graph_inputs(hv: np.ndarray, tokens: List[int], positions: List[int], tables: List[List[int]],
                           Bb: int, Wb: int, pad_block: int, bs: int) -> None:
        """Fill the int32 staging buffer of a (Bb, Wb) decode graph: tokens, positions, context lengths,
        slot blocks, slot offsets ([Bb] each), then the [Bb, Wb] block tables.  Rows past the real batch
        decode token 0 at position 0 with a one-token context in ``pad_block``."""
        B = len(tokens)
        hv[:5 * Bb + Bb * Wb] = 0
        pos = np.asarray(positions, dtype=np.int64)
        hv[:B] = np.asarray(tokens, dtype=np.int64)
        hv[Bb:Bb + B] = pos
        hv[2 * Bb:3 * Bb] = 1
        hv[2 * Bb:2 * Bb + B] = pos + 1
        hv[3 * Bb:4 * Bb] = pad_block
        hv[4 * Bb:4 * Bb + B] = pos % bs
        grid = hv[5 * Bb:5 * Bb + Bb * Wb].reshape(Bb, Wb)
        grid[:, 0] = pad_block
        for b, t in enumerate(tables):
            grid[b, :len(t)] = t
        hv[3 * Bb:3 * Bb + B] = grid[np.arange(B), pos // bs]

    def reset_graphs(self) -> None:
        """Drop the captured decode graphs (they are captured again on use)."""
        self._graphs.clear()
        self._graph_fail.clear()

    def _capture(self, Bb: int, Wb: int) -> Optional[Dict[str, Any]]:
        """Capture the decode step of a (batch, width) bucket; None if the model cannot be captured."""
        from rl_project_b200.models.attention.causal import PagedDecodeMeta

        dev = self.device
        # the RoPE tables must not grow (reallocate) inside the graph: size them for the longest sequence
        for blk in self.model.transformer.h:
            rope = getattr(getattr(blk, "attn", None), "rope", None)
            if rope is not None:
                rope.tables(self.max_seq_len + 1, dev)
        buf = torch.zeros(5 * Bb + Bb * Wb, dtype=torch.int32, device=dev)
        buf[2 * Bb:3 * Bb] = 1  # padding rows: context of one token...
        buf[3 * Bb:4 * Bb] = self._pad_block  # ...written into the padding block
        buf[5 * Bb:].view(Bb, Wb)[:, 0] = self._pad_block
        meta = PagedDecodeMeta(positions=buf[Bb:2 * Bb].view(Bb, 1), max_pos=self.max_seq_len - 1,
                               ctx_lens=buf[2 * Bb:3 * Bb], slot_block=buf[3 * Bb:4 * Bb], slot_off=buf[4 * Bb:5 * Bb],
                               block_tables=buf[5 * Bb:].view(Bb, Wb),
                               split_tokens=self._split_tokens(Bb, Wb * self.allocator.block_size))
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        try:
            with torch.cuda.stream(side):  # warm-up: lazy allocations and one-time set-up happen outside capture
                for _ in range(2):
                    self.model.decode_paged(buf[:Bb].long(), self.kv, meta)
            cur.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self._graph_pool):
                logits = self.model.decode_paged(buf[:Bb].long(), self.kv, meta)
        except Exception as exc:  # noqa: BLE001 - e.g. a host synchronisation inside the model's decode
            torch.cuda.synchronize(dev)
            log.warning("decode_graph_capture_failed", batch=Bb, width=Wb, error=repr(exc))
            return None
        if self._graph_pool is None:
            self._graph_pool = graph.pool()
        return {"graph": graph, "buf": buf, "logits": logits}

    def _decode_graph(self, seqs: List[_Seq]) -> Optional[int]:
        """The paged decode step replayed from a captured graph; None when no graph serves this bucket."""
        B = len(seqs)
        bs = self.allocator.block_size
        tables = [self.allocator.tables[s.req.id] for s in seqs]
        width = max(len(t) for t in tables)
        Bb = self._pow2(B, self.max_batch)
        Wb = self._pow2(width, (self.max_seq_len + bs - 1) // bs + 1)
        key = (Bb, Wb)
        if key in self._graph_fail:
            return None
        gr = self._graphs.get(key)
        if gr is None:
            gr = self._capture(Bb, Wb)
            if gr is None:
                self._graph_fail.add(key)
                return None
            self._graphs[key] = gr
        n = 5 * Bb + Bb * Wb
        if self._pinned is None or self._pinned.numel() < n:
            self._pinned = torch.empty(max(n, 1024), dtype=torch.int32, pin_memory=True)
        host = self._pinned[:n]
        self.stage_graph_inputs(host.numpy(), [s.tokens[-1] for s in seqs], [s.position for s in seqs], tables,
                                Bb, Wb, self._pad_block, bs)
        gr["buf"].copy_(host, non_blocking=True)
        with self.tracer.span("decode", batch=B, graph=1):
            gr["graph"].replay()
        self.decode_steps += 1
        for s in seqs:
            s.position += 1
        return self._sample_and_emit(seqs, gr["logits"][:B], None)

    def _split_tokens(self, B: int, max_ctx: int) -> int:
        """Split long contexts over several CTAs when the batch alone cannot fill the GPU."""
        if self.device.type != "cuda" or max_ctx <= 256:
            return 0
        ctas = B * self.model.kv_layout()[1]
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
            produced += self._sample_and_emit(group, logits)
        return produced

    # ------------------------------------------------------------ sampling
    @staticmethod
    def _plain(p: SamplingParams) -> bool:
        """Temperature-only sampling: the fused sampler's domain."""
        return (not p.top_k) and p.top_p in (None, 1.0) and not p.min_p and p.repetition_penalty == 1.0

    def _sample_and_emit(self, seqs: List[_Seq], logits: torch.Tensor, evs: Optional[List[Any]] = None) -> int:
        B = len(seqs)
        if evs is not None:
            evs.append(self._event())
        self._sample_calls += 1
        # the step's sampling seed comes from torch's host generator, so a checkpoint's RNG state (which
        # holds that generator) also fixes every sample drawn after a resume
        seed = int(torch.randint(0, 1 << 62, (1,)).item())
        out = torch.empty(B, dtype=torch.long, device=logits.device)
        fused = [i for i, s in enumerate(seqs) if self._plain(s.req.params)] if logits.is_cuda else []
        if fused:
            from rl_project_b200.ops.sampling import sample_tokens

            temps = torch.tensor([seqs[i].req.params.temperature for i in fused], dtype=torch.float32)
            if len(fused) == B:
                out, _ = sample_tokens(logits, temps.to(logits.device, non_blocking=True), seed)
            else:
                idx = torch.as_tensor(fused, device=logits.device)
                tok, _ = sample_tokens(logits.index_select(0, idx), temps.to(logits.device), seed)
                out.index_copy_(0, idx, tok)
        fused_set = set(fused)
        groups: Dict[tuple, List[int]] = defaultdict(list)
        for i, s in enumerate(seqs):
            if i in fused_set:
                continue
            p = s.req.params
            if p.repetition_penalty != 1.0:
                f = apply_sampling_filters(logits[i:i + 1].float(), p.temperature, p.top_k, p.top_p, p.min_p,
                                           p.repetition_penalty, s.tokens)
                out[i] = sample_from_logits(f, p.temperature).view(())
            else:
                groups[p.filter_key()].append(i)
        for (temp, top_k, top_p, min_p), rows in groups.items():
            idx = torch.as_tensor(rows, device=logits.device)
            sub = (logits if len(rows) == B else logits.index_select(0, idx)).float()
            if temp <= 0:
                tok = sub.argmax(-1)
            else:
                tok = sample_from_logits(apply_sampling_filters(sub, temp, top_k, top_p, min_p), temp).view(-1)
            if len(rows) == B:
                out = tok
            else:
                out.index_copy_(0, idx, tok)
        if evs is not None:
            evs.append(self._event())
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
               "decode_graphs": len(self._graphs) if self.decode_graphs else 0, "spans": self.tracer.summary()}
        if self.kv is not None:
            out["kv_cache_bytes"] = self.kv.nbytes
        return out
