"""Host-side liveness of tensor-parallel ranks through the rendezvous store.

Every rank runs a daemon thread that writes `<prefix>/<rank>` =
"<wall time>:<step>" into the torch.distributed key-value store every
`interval_s`.  A monitor thread (on every rank) reads the peers' keys and
calls `on_lost(rank, reason)` once when a peer's beat is older than
`stale_s` (the process died or its host thread stopped) or when its step
counter trails this rank's by more than `max_step_lag` for longer than
`stale_s` (its engine is stuck while this rank advances).  Detection needs
no collective and no GPU, so it also works while the lockstep exchange is
blocked waiting for the lost rank.

The serving runtime (server/runtime.py) fails every in-flight request with
the reason and refuses new ones.  The reference has no multi-rank liveness
(its collectives are no-ops, crates/engine/src/core/parallelism.rs:105-178);
its server exposes only process readiness.
"""
from __future__ import annotations

import threading
import time
from typing import Callable, Dict, Optional


class Heartbeat:
    def __init__(self, store, rank: int, world: int, on_lost: Callable[[int, str], None], interval_s: float = 0.5,
                 stale_s: float = 10.0, max_step_lag: int = 2, prefix: str = "bloom/hb"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.on_lost = on_lost
        self.interval_s, self.stale_s, self.max_step_lag = float(interval_s), float(stale_s), int(max_step_lag)
        self.prefix = prefix
        self.step = 0
        self.lost: Dict[int, str] = {}
        self._stop = threading.Event()
        self._first_seen: Dict[int, float] = {}
        self._lag_since: Dict[int, float] = {}
        self._threads = [threading.Thread(target=self._beat, name="bloom-heartbeat", daemon=True),
                         threading.Thread(target=self._watch, name="bloom-heartbeat-watch", daemon=True)]

    def start(self) -> "Heartbeat":
        self._write()
        for t in self._threads:
            t.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        for t in self._threads:
            if t.is_alive() and t is not threading.current_thread():
                t.join(timeout=2 * self.interval_s + 1.0)

    def tick(self) -> None:
        """Called by the engine loop after every step."""
        self.step += 1

    # ---------------------------------------------------------------- threads
    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _write(self) -> None:
        self.store.set(self._key(self.rank), f"{time.time():.6f}:{self.step}")

    def _beat(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self._write()
            except Exception:  # the store's host (rank 0) is gone: the watcher reports it
                pass

    def read(self, r: int) -> Optional[tuple]:
        k = self._key(r)
        if not self.store.check([k]):
            return None
        t, s = self.store.get(k).decode().split(":")
        return float(t), int(s)

    def _declare(self, r: int, reason: str) -> None:
        if r in self.lost:
            return
        self.lost[r] = reason
        self.on_lost(r, reason)

    def check(self, now: Optional[float] = None) -> None:
        """One pass of the watcher (also callable directly)."""
        now = time.time() if now is None else now
        for r in range(self.world):
            if r == self.rank or r in self.lost:
                continue
            try:
                beat = self.read(r)
            except Exception as e:  # store unreachable: rank 0 (its host) is gone
                self._declare(r, f"rank {r} unreachable through the store: {e}")
                continue
            if beat is None:
                first = self._first_seen.setdefault(r, now)
                if now - first > self.stale_s:
                    self._declare(r, f"rank {r} never sent a heartbeat within {self.stale_s:.0f} s")
                continue
            t, step = beat
            if now - t > self.stale_s:
                self._declare(r, f"rank {r} heartbeat is {now - t:.1f} s old")
                continue
            if self.step - step > self.max_step_lag:
                since = self._lag_since.setdefault(r, now)
                if now - since > self.stale_s:
                    self._declare(r, f"rank {r} is stuck at step {step} while rank {self.rank} is at {self.step}")
            else:
                self._lag_since.pop(r, None)

    def _watch(self) -> None:
        while not self._stop.wait(self.interval_s):
            self.check()
