"""Rank-failure detection on the host: heartbeats through a key-value store.

The reference configures no timeout, watchdog or rank-failure detection
(``src/forgeline/distributed/runtime.py:48-55`` calls ``init_process_group``
without a timeout).  Here every process group gets an explicit timeout
(``parallel/runtime.py``), every device-side wait of the fused kernels is
bounded, and :class:`HeartbeatMonitor` lets the ranks learn that a peer is
gone *between* steps, before they launch the next collective:

* a daemon thread on each rank writes ``<prefix>/<rank>`` = a monotonically
  increasing beat count every ``interval_s`` to a store shared by the job (the
  process group's TCP store, or any ``torch.distributed.Store``);
* ``check()`` -- called by the trainer before a step -- reads every peer's
  count; a peer whose count has not advanced for ``timeout_s`` seconds (or that
  announced ``stop``) is reported by raising ``DistributedTimeoutError`` naming
  it, so the surviving ranks leave the step loop with a clear error instead of
  blocking inside a collective;
* ``stop(reason)`` marks a clean departure (``<prefix>/<rank>/left``) so peers
  can tell an orderly exit from a crash.

The counts, not wall-clock times, are compared, so hosts need no synchronised
clocks.  Recovery is resuming from the last atomic checkpoint.
"""

from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional

import torch.distributed as dist

from rl_project_b200.core.errors import DistributedTimeoutError


class HeartbeatMonitor:
    def __init__(self, store: "dist.Store", rank: int, world: int, interval_s: float = 0.5,
                 timeout_s: float = 10.0, prefix: str = "rlb_hb"):
        self.store = store
        self.rank, self.world = int(rank), int(world)
        self.interval_s, self.timeout_s = float(interval_s), float(timeout_s)
        self.prefix = prefix
        self._beats = 0
        self._stop = threading.Event()
        self._seen: Dict[int, tuple] = {}  # peer -> (last count, local time it last changed)
        self._thread: Optional[threading.Thread] = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def start(self) -> "HeartbeatMonitor":
        try:  # a departure mark left in a store that outlived an earlier run of this rank
            self.store.delete_key(f"{self._key(self.rank)}/left")
        except Exception:
            pass
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def _beat(self) -> None:
        self._beats += 1
        self.store.set(self._key(self.rank), str(self._beats))

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
            except Exception:  # store gone (job shutting down): stop beating
                return

    def stop(self, reason: str = "done") -> None:
        """Stop beating and tell the peers this rank left on purpose."""
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval_s + 1)
        try:
            self.store.set(f"{self._key(self.rank)}/left", reason)
        except Exception:
            pass

    def _count(self, r: int) -> Optional[int]:
        try:
            if not self.store.check([self._key(r)]):
                return None
            return int(self.store.get(self._key(r)))
        except Exception:
            return None

    def _left(self, r: int) -> Optional[str]:
        try:
            if self.store.check([f"{self._key(r)}/left"]):
                return self.store.get(f"{self._key(r)}/left").decode()
        except Exception:
            pass
        return None

    def dead_peers(self) -> List[int]:
        """Peers that left or whose beat count has not advanced for ``timeout_s`` (never seen counts as 0)."""
        now = time.monotonic()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            if self._left(r) is not None:
                dead.append(r)
                continue
            c = self._count(r)
            prev = self._seen.get(r)
            if prev is None or c != prev[0]:
                self._seen[r] = (c, now)
            elif now - prev[1] > self.timeout_s:
                dead.append(r)
        return dead

    def check(self) -> None:
        """Raise for gone peers.  Rate-limited to one store pass per ``interval_s`` (cheap per step)."""
        now = time.monotonic()
        if now - getattr(self, "_last_check", -1e9) < self.interval_s:
            return
        self._last_check = now
        dead = self.dead_peers()
        if dead:
            reasons = {r: self._left(r) for r in dead}
            desc = ", ".join(f"rank {r}" + (f" (left: {reasons[r]})" if reasons[r] else " (no heartbeat)")
                             for r in dead)
            raise DistributedTimeoutError(f"peer ranks are gone: {desc}",
                                          hint="Restart the job; it resumes from the last checkpoint.")

    def wait_all_alive(self, timeout_s: Optional[float] = None) -> None:
        """Block until every peer has beaten at least once (a rank that never joins raises after the limit)."""
        limit = time.monotonic() + (timeout_s if timeout_s is not None else self.timeout_s)
        while True:
            missing = [r for r in range(self.world) if r != self.rank and self._count(r) is None]
            if not missing:
                return
            if time.monotonic() > limit:
                raise DistributedTimeoutError(f"ranks never joined: {missing}",
                                              hint="Check the launcher: every rank must start.")
            time.sleep(min(self.interval_s, 0.1))


def monitor_for_process_group(interval_s: float = 0.5, timeout_s: float = 10.0) -> Optional[HeartbeatMonitor]:
    """A started monitor on the default process group's store (None when not distributed)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return None
    from torch.distributed.distributed_c10d import _get_default_store

    return HeartbeatMonitor(_get_default_store(), dist.get_rank(), dist.get_world_size(), interval_s,
                            timeout_s).start()


def attach(strategy, cfg) -> None:
    """Give ``strategy`` a started monitor (from ``cfg.heartbeat_*``) and a ``check_health`` method."""
    iv = float(getattr(cfg, "heartbeat_interval_s", 0.0) or 0.0)
    strategy.monitor = monitor_for_process_group(iv, float(getattr(cfg, "heartbeat_timeout_s", 60.0))) \
        if iv > 0 else None


def detach(strategy) -> None:
    m = getattr(strategy, "monitor", None)
    if m is not None:
        m.stop("teardown")
        strategy.monitor = None
