"""Admission control of the paged inference engine (continuous batching).

Each ``admit()`` call forms the next prefill batch for the engine's step.  Requests wait in arrival order
and the queue head is never overtaken, so a long prompt cannot be starved by short ones behind it.  The
head is taken while

* the running set has a free slot (``max_batch``),
* the batch's prompt tokens stay within ``prefill_token_budget`` (one batched prefill sized so the
  decode of the running set is not stalled for long; the first request of a batch is always allowed), and
* the paged KV allocator can hold its prompt plus the first generated token.

A request that can never fit (prompt plus ``max_tokens`` beyond ``max_seq_len``) fails at the head
without blocking the rest.  Cancelling a waiting request finishes it at once; a running one is flagged
and the engine retires it at its next token.  Behaviour matches the reference's scheduler
(``src/forgeline/inference/scheduler.py:14-75``) where it defines one: FIFO, the length rejection, waiting
for blocks, cancellation.
"""

from __future__ import annotations

import threading
from collections import Counter, OrderedDict
from typing import Dict, List, Optional

from rl_project_b200.inference.paged_memory import PagedBlockAllocator
from rl_project_b200.inference.requests import GenerationRequest


class Scheduler:
    def __init__(self, allocator: PagedBlockAllocator, max_batch: int = 8, max_seq_len: int = 512,
                 prefill_token_budget: Optional[int] = None):
        self.allocator = allocator
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.prefill_token_budget = prefill_token_budget
        self._waiting: "OrderedDict[str, GenerationRequest]" = OrderedDict()
        self._active: Dict[str, GenerationRequest] = {}
        self._tally: Counter = Counter()
        self._mu = threading.Lock()

    # ------------------------------------------------------------ views
    @property
    def pending(self) -> List[GenerationRequest]:
        with self._mu:
            return list(self._waiting.values())

    @property
    def running(self) -> Dict[str, GenerationRequest]:
        with self._mu:
            return dict(self._active)

    @property
    def completed(self) -> int:
        return self._tally["completed"]

    @property
    def rejected(self) -> int:
        return self._tally["rejected"]

    # ------------------------------------------------------------ queue
    def submit(self, req: GenerationRequest) -> None:
        with self._mu:
            self._waiting[req.id] = req

    def _never_fits(self, req: GenerationRequest) -> Optional[str]:
        need = len(req.prompt_tokens) + req.params.max_tokens
        if need > self.max_seq_len:
            return f"prompt+max_tokens {need} exceeds max_seq_len {self.max_seq_len}"
        return None

    def admit(self) -> List[GenerationRequest]:
        batch: List[GenerationRequest] = []
        prompt_tokens = 0
        with self._mu:
            while self._waiting and len(self._active) < self.max_batch:
                rid, req = next(iter(self._waiting.items()))
                why = self._never_fits(req)
                if why is not None:
                    del self._waiting[rid]
                    self._tally["rejected"] += 1
                    req.finish("length", error=why)
                    continue
                n = len(req.prompt_tokens)
                if batch and self.prefill_token_budget is not None and prompt_tokens + n > self.prefill_token_budget:
                    break  # the rest waits for the next step's prefill
                if not self.allocator.can_allocate(rid, n + 1):
                    break  # head of line waits until blocks are freed
                del self._waiting[rid]
                self.allocator.allocate(rid, n)
                req.start()
                self._active[rid] = req
                batch.append(req)
                prompt_tokens += n
        return batch

    def retire(self, req: GenerationRequest, reason: str, error: Optional[str] = None) -> None:
        with self._mu:
            if self._active.pop(req.id, None) is not None:
                self.allocator.free(req.id)
            self._tally["completed"] += 1
        req.finish(reason, error)

    def cancel(self, request_id: str) -> bool:
        with self._mu:
            waiting = self._waiting.pop(request_id, None)
            if waiting is None:
                active = self._active.get(request_id)
                if active is None:
                    return False
                active.meta["cancel"] = True  # the engine retires it at its next token
                return True
        waiting.finish("cancelled")
        return True

    def has_work(self) -> bool:
        with self._mu:
            return bool(self._waiting) or bool(self._active)

    def stats(self) -> Dict[str, float]:
        with self._mu:
            out = {"pending": len(self._waiting), "running": len(self._active),
                   "completed": self._tally["completed"], "rejected": self._tally["rejected"]}
        out.update(self.allocator.stats())
        return out
