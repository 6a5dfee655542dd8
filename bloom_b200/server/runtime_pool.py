"""Multi-model residency for the HTTP server.

RuntimePool
    Loaded runtimes (pipeline + serving runtime) keyed by model id, oldest
    first.  One entry is the default (requests that name no model, or the
    served id).  Publishing into a full pool evicts the oldest non-default
    entry; a same-key publication replaces the old generation.  Retired
    entries are returned to the caller, which shuts them down outside the
    pool lock.  Reference: crates/server/src/runtime_pool.rs:26-160.

MemoryBudget / MemoryPermit
    Aggregate host and device byte limits over every resident runtime.  A
    runtime is published only with a permit for its footprint (the
    manifest's memory estimate, or what loading measured); a permit is
    released when its runtime retires.  `evaluate` reports whether a
    candidate would fit without reserving anything.  Reference:
    crates/server/src/runtime_memory.rs:13-260.

Keep-alive (Ollama residency)
    `parse_keep_alive` reads Ollama's keep_alive (seconds as a number, or a
    duration string such as "5m", "1h30m", "250ms"; negative = stay
    resident, 0 = unload after the request, default 5 minutes, at most 365
    days).  An entry's deadline is (re)armed when a request that named it
    finishes; `expired(now)` lists entries whose deadline passed.
    Reference: crates/server/src/ollama.rs:185-400, 2689-2780.
"""
from __future__ import annotations

import re
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

DEFAULT_KEEP_ALIVE_S = 300.0
MAX_KEEP_ALIVE_S = 365 * 24 * 3600.0
INDEFINITE = -1.0  # keep_alive value: stay resident


class KeepAliveError(ValueError):
    pass


_UNITS = {"ns": 1e-9, "us": 1e-6, "µs": 1e-6, "ms": 1e-3, "s": 1.0, "m": 60.0, "h": 3600.0}
_PART = re.compile(r"(\d+(?:\.\d*)?|\.\d+)(ns|us|µs|ms|s|m|h)")


def parse_keep_alive(value: Any) -> float:
    """-> seconds; INDEFINITE (-1) to stay resident; 0 to unload now."""
    if value is None:
        return DEFAULT_KEEP_ALIVE_S
    if isinstance(value, bool):
        raise KeepAliveError("keep_alive must be a number or duration string")
    if isinstance(value, (int, float)):
        secs = float(value)
    elif isinstance(value, str):
        v = value.strip()
        if not v or len(v) > 128:
            raise KeepAliveError("keep_alive duration string is empty or too long")
        try:
            secs = float(v)
        except ValueError:
            sign = -1.0 if v[0] == "-" else 1.0
            body = v[1:] if v[0] in "+-" else v
            pos, total = 0, 0.0
            for m in _PART.finditer(body):
                if m.start() != pos:
                    raise KeepAliveError("keep_alive duration string is invalid") from None
                total += float(m.group(1)) * _UNITS[m.group(2)]
                pos = m.end()
            if pos != len(body) or pos == 0:
                raise KeepAliveError("keep_alive duration string is invalid") from None
            secs = sign * total
    else:
        raise KeepAliveError("keep_alive must be a number or duration string")
    if secs != secs or secs in (float("inf"), float("-inf")):
        raise KeepAliveError("keep_alive must be finite")
    if secs < 0:
        return INDEFINITE
    if secs > MAX_KEEP_ALIVE_S:
        raise KeepAliveError("keep_alive cannot exceed 365 days")
    return secs


# ---------------------------------------------------------------- memory permits
@dataclass(frozen=True)
class Footprint:
    host_bytes: int = 0
    device_bytes: int = 0

    def __add__(self, o: "Footprint") -> "Footprint":
        return Footprint(self.host_bytes + o.host_bytes, self.device_bytes + o.device_bytes)

    def __sub__(self, o: "Footprint") -> "Footprint":
        return Footprint(self.host_bytes - o.host_bytes, self.device_bytes - o.device_bytes)


class MemoryError_(RuntimeError):
    """A runtime does not fit the aggregate memory budget (HTTP 507)."""


class MemoryBudget:
    def __init__(self, host_limit_bytes: int, device_limit_bytes: int):
        self.limit = Footprint(int(host_limit_bytes), int(device_limit_bytes))
        self.used = Footprint()
        self.generations = 0
        self._lock = threading.Lock()

    def _check(self, fp: Footprint, available: Optional[Footprint]) -> Optional[str]:
        if fp.host_bytes < 0 or fp.device_bytes < 0:
            return "negative memory footprint"
        if available is not None:
            if fp.host_bytes > available.host_bytes:
                return (f"needs {fp.host_bytes} host bytes but only {available.host_bytes} are free")
            if fp.device_bytes > available.device_bytes:
                return (f"needs {fp.device_bytes} device bytes but only {available.device_bytes} are free")
        nxt = self.used + fp
        if nxt.host_bytes > self.limit.host_bytes:
            return f"host memory budget {self.limit.host_bytes} would be exceeded ({nxt.host_bytes})"
        if nxt.device_bytes > self.limit.device_bytes:
            return f"device memory budget {self.limit.device_bytes} would be exceeded ({nxt.device_bytes})"
        return None

    def evaluate(self, fp: Footprint, available: Optional[Footprint] = None) -> Tuple[bool, Optional[str], Dict]:
        with self._lock:
            why = self._check(fp, available)
            return why is None, why, self._snapshot()

    def reserve(self, fp: Footprint, available: Optional[Footprint] = None) -> "MemoryPermit":
        with self._lock:
            why = self._check(fp, available)
            if why is not None:
                raise MemoryError_(why)
            self.used = self.used + fp
            self.generations += 1
            return MemoryPermit(self, fp)

    def _release(self, fp: Footprint) -> None:
        with self._lock:
            self.used = self.used - fp
            self.generations -= 1

    def _snapshot(self) -> Dict:
        return {"host_limit_bytes": self.limit.host_bytes, "host_used_bytes": self.used.host_bytes,
                "device_limit_bytes": self.limit.device_bytes, "device_used_bytes": self.used.device_bytes,
                "generations": self.generations}

    def snapshot(self) -> Dict:
        with self._lock:
            return self._snapshot()


class MemoryPermit:
    def __init__(self, budget: MemoryBudget, fp: Footprint):
        self.budget = budget
        self.footprint = fp
        self._released = False

    def resize(self, fp: Footprint) -> None:
        """Replace the estimate by what loading measured (growth must still fit)."""
        b = self.budget
        with b._lock:
            grow = Footprint(max(0, fp.host_bytes - self.footprint.host_bytes),
                             max(0, fp.device_bytes - self.footprint.device_bytes))
            why = b._check(grow, None)
            if why is not None:
                raise MemoryError_(why)
            b.used = b.used - self.footprint + fp
            self.footprint = fp

    def release(self) -> None:
        if not self._released:
            self._released = True
            self.budget._release(self.footprint)


# ---------------------------------------------------------------- pool
@dataclass
class RuntimeEntry:
    key: str
    source: str
    pipeline: Any
    runtime: Any
    permit: Optional[MemoryPermit] = None
    created: float = field(default_factory=time.time)
    last_used: float = field(default_factory=time.time)
    # residency deadline after each request: INDEFINITE unless an Ollama
    # request (or the operator's load call) gave a keep_alive
    keep_alive_s: float = INDEFINITE
    expires_at: Optional[float] = None  # wall clock; None = no deadline armed

    @property
    def active(self) -> int:
        """Requests being served by this runtime right now."""
        return int(getattr(self.runtime, "in_flight", 0) or 0)

    on_retire: List[Any] = field(default_factory=list)  # callbacks (key) run after shutdown

    def retire(self) -> None:
        try:
            self.runtime.shutdown()
        finally:
            if self.permit is not None:
                self.permit.release()
                self.permit = None
            for cb in self.on_retire:
                cb(self.key)
            self.on_retire = []


class RuntimePool:
    def __init__(self, capacity: int = 1):
        if capacity < 1:
            raise ValueError("runtime pool capacity must be at least 1")
        self.capacity = int(capacity)
        self._entries: "OrderedDict[str, RuntimeEntry]" = OrderedDict()
        self.default_key: Optional[str] = None
        self._lock = threading.Lock()

    def __len__(self) -> int:
        return len(self._entries)

    def publish(self, entry: RuntimeEntry, make_default: bool = False) -> List[RuntimeEntry]:
        """Insert (or replace) an entry; returns retired entries (replaced
        generation first, then capacity victims, oldest non-default first)."""
        retired: List[RuntimeEntry] = []
        with self._lock:
            old = self._entries.pop(entry.key, None)
            if old is not None:
                retired.append(old)
            if make_default:
                self.default_key = entry.key
            while len(self._entries) >= self.capacity:
                victim = next((k for k in self._entries if k != self.default_key), None)
                if victim is None:  # capacity one: the previous default goes
                    victim = next(iter(self._entries))
                retired.append(self._entries.pop(victim))
            self._entries[entry.key] = entry
            if self.default_key is None or self.default_key not in self._entries:
                self.default_key = entry.key
        return retired

    def get(self, key: str) -> Optional[RuntimeEntry]:
        with self._lock:
            return self._entries.get(key)

    def select(self, name: Optional[str]) -> Optional[RuntimeEntry]:
        """The entry a request's `model` field names (exact id, or an id that
        ends with it, e.g. a tag without its path); None names the default."""
        with self._lock:
            if not name:
                return self._entries.get(self.default_key) if self.default_key else None
            if name in self._entries:
                return self._entries[name]
            for k, e in self._entries.items():
                if k.endswith(str(name)):
                    return e
            return None

    def remove(self, key: str) -> Optional[RuntimeEntry]:
        with self._lock:
            e = self._entries.pop(key, None)
            if key == self.default_key:
                self.default_key = next(iter(self._entries), None)
            return e

    def evict_for(self, budget: MemoryBudget, fp: Footprint, protect: Optional[str] = None) -> List[RuntimeEntry]:
        """Remove least recently used idle non-default entries until `fp` fits."""
        retired: List[RuntimeEntry] = []
        while not budget.evaluate(fp)[0]:
            with self._lock:
                cands = [e for k, e in self._entries.items()
                         if k not in (self.default_key, protect) and e.active == 0]
                if not cands:
                    break
                v = min(cands, key=lambda e: e.last_used)
                self._entries.pop(v.key)
            v.retire()
            retired.append(v)
        return retired

    def touch(self, key: str, keep_alive_s: Optional[float] = None) -> None:
        """A request that used `key` finished: record it and (re)arm the deadline."""
        with self._lock:
            e = self._entries.get(key)
            if e is None:
                return
            e.last_used = time.time()
            if keep_alive_s is not None:
                e.keep_alive_s = keep_alive_s
            e.expires_at = None if e.keep_alive_s == INDEFINITE else e.last_used + e.keep_alive_s

    def expired(self, now: Optional[float] = None) -> List[str]:
        now = time.time() if now is None else now
        with self._lock:
            return [k for k, e in self._entries.items()
                    if e.expires_at is not None and e.expires_at <= now and e.active == 0]

    def entries(self) -> List[RuntimeEntry]:
        with self._lock:
            return list(self._entries.values())
