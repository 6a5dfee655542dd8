"""Host-side tracing spans: `with span("engine.step", tokens=T): ...`.

Every span is timed with the monotonic clock and, when enabled:
  * logged at DEBUG level on the "bloom_b200.trace" logger (name, fields, ms);
  * pushed as an NVTX range (BLOOM_NVTX=1) so a GPU timeline shows the
    engine's phases around its kernels;
  * appended as a Chrome trace event (BLOOM_TRACE=<file.json>; open it in
    chrome://tracing or Perfetto), written by `flush()` and at exit.
With none of them enabled a span costs two clock reads.  Span names used by
the engine: model.load, engine.step, engine.schedule, engine.forward,
engine.sample, pipeline.run, server.request.  Reference: tracing spans
around load / run / prefill / decode (crates/engine/src/core/pipeline.rs:89-95,
executor/candle.rs:2261-2262).
"""
from __future__ import annotations

import atexit
import json
import logging
import os
import threading
import time
from contextlib import contextmanager
from typing import Dict, List

log = logging.getLogger("bloom_b200.trace")
_NVTX = os.environ.get("BLOOM_NVTX", "0") == "1"
_TRACE_PATH = os.environ.get("BLOOM_TRACE", "")
_events: List[Dict] = []
_lock = threading.Lock()
_t0 = time.perf_counter()
_stats: Dict[str, List[float]] = {}


def enabled() -> bool:
    return _NVTX or bool(_TRACE_PATH) or log.isEnabledFor(logging.DEBUG)


@contextmanager
def span(name: str, **fields):
    t = time.perf_counter()
    nv = None
    if _NVTX:
        try:
            import torch

            torch.cuda.nvtx.range_push(name)
            nv = torch.cuda.nvtx
        except Exception:
            nv = None
    try:
        yield
    finally:
        dt = time.perf_counter() - t
        if nv is not None:
            nv.range_pop()
        with _lock:
            st = _stats.setdefault(name, [0, 0.0])
            st[0] += 1
            st[1] += dt
            if _TRACE_PATH:
                _events.append({"name": name, "ph": "X", "ts": (t - _t0) * 1e6, "dur": dt * 1e6, "pid": os.getpid(),
                                "tid": threading.get_ident() & 0xFFFF, "args": fields})
        if log.isEnabledFor(logging.DEBUG):
            log.debug("%s %.3f ms %s", name, dt * 1e3, fields or "")


def stats() -> Dict[str, Dict[str, float]]:
    """Count and total seconds per span name since start."""
    with _lock:
        return {k: {"count": int(v[0]), "seconds": round(v[1], 6)} for k, v in _stats.items()}


def flush(path: str = "") -> str:
    path = path or _TRACE_PATH
    if not path:
        return ""
    with _lock:
        ev = list(_events)
    with open(path, "w") as f:
        json.dump({"traceEvents": ev, "displayTimeUnit": "ms"}, f)
    return path


if _TRACE_PATH:
    atexit.register(flush)
