"""Serving runtime: one engine thread drives in-flight batching for every HTTP request.

HTTP handlers call `submit()` and consume an async stream of token ids; the
engine thread admits new requests into the C++ scheduler between steps, runs
`LLMEngine.step()` (one batched forward for all running requests) and pushes
each new token to its request's asyncio queue.  Detokenisation and stop-string
filtering run on the handler side, so the engine loop never waits on Python
text work.  Cancellation (client disconnect, /v1/cancel/{id}) aborts the
request in the scheduler before the next step, which frees its KV blocks.

The reference's IFB path instead kept a separate model wrapper per request and
looped over them one at a time (crates/server/src/lib.rs:2796-3063, worker
loop stepping every 5 ms); CPU and echo pipelines here keep that simpler
one-request-at-a-time execution in a worker thread.
"""
from __future__ import annotations

import asyncio
import itertools
import logging
import os
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

log = logging.getLogger("bloom_b200.server.runtime")

_ids = itertools.count(1)


@dataclass
class StreamItem:
    token: Optional[int] = None
    text: Optional[str] = None  # used by non-engine pipelines (already detokenised)
    finished: bool = False
    reason: Optional[str] = None
    error: Optional[str] = None


@dataclass
class Submission:
    id: str
    prompt_ids: List[int]
    params: Any
    loop: asyncio.AbstractEventLoop
    queue: asyncio.Queue
    created: float = field(default_factory=time.time)
    engine_rid: Optional[int] = None
    cancelled: bool = False
    first_token_at: Optional[float] = None
    last_token_at: Optional[float] = None
    n_tokens: int = 0
    messages: Any = None
    segment: int = 0  # 0 foreground, 1 realtime stream, 2 background batch, 3 maintenance


class TPControl:
    """Keeps the engines of tensor-parallel ranks in lockstep.  Rank 0 (the
    HTTP process) publishes, before every engine step, the requests it admits
    and aborts; the other ranks apply the same calls in the same order (so the
    replicated C++ schedulers assign the same ids and schedule the same rows)
    and step with it.  Messages travel over a gloo (CPU) process group; an
    idle rank 0 sends an empty message every second.  Independently, every
    rank beats into the rendezvous store (parallel/heartbeat.py), so a rank
    that died or stopped stepping is noticed within BLOOM_HEARTBEAT_STALE_S
    (default 10 s) even while the exchange is blocked on it."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group if group is not None else dist.new_group(backend="gloo")
        self.rank = dist.get_rank()
        self.heartbeat = None

    def start_heartbeat(self, on_lost) -> None:
        from ..parallel.heartbeat import Heartbeat

        store = self.dist.distributed_c10d._get_default_store()
        self.heartbeat = Heartbeat(store, self.rank, self.dist.get_world_size(), on_lost,
                                   stale_s=float(os.environ.get("BLOOM_HEARTBEAT_STALE_S", "10"))).start()

    def tick(self) -> None:
        if self.heartbeat is not None:
            self.heartbeat.tick()

    def exchange(self, msg=None):
        obj = [msg]
        self.dist.broadcast_object_list(obj, src=0, group=self.group)
        return obj[0]


def follower_loop(engine, ctrl: TPControl) -> None:
    """Ranks > 0: apply rank 0's admissions / aborts and step in lockstep.
    If rank 0 is gone, the exchange raises (connection closed, or the process
    group's timeout) and so does this loop: the rank exits with an error
    instead of waiting for a leader that never speaks again."""
    if getattr(ctrl, "heartbeat", None) is None and hasattr(ctrl, "start_heartbeat"):
        ctrl.start_heartbeat(lambda r, why: log.error("tensor-parallel rank lost: %s", why))
    while True:
        msg = ctrl.exchange(None)
        if msg.get("stop"):
            if getattr(ctrl, "heartbeat", None) is not None:
                ctrl.heartbeat.stop()
            return
        for prompt, params, prio in msg.get("add", []):
            engine.add_request(prompt, params, prio)
        for rid in msg.get("abort", []):
            engine.abort(rid)
        if msg.get("step"):
            for r in engine.step():
                if r.finished:
                    engine.requests.pop(r.request_id, None)
            if hasattr(ctrl, "tick"):
                ctrl.tick()


# request class -> engine scheduler priority (higher first); classes follow the
# reference's BloomScheduler (scheduler/mod.rs:893-915): foreground interactive
# > realtime stream > background batch > maintenance
SEGMENT_PRIORITY = {0: 3, 1: 2, 2: 1, 3: 0}
SEGMENTS = {"foreground": 0, "realtime": 1, "background": 2, "maintenance": 3}


class ThermalMonitor:
    """Reads the GPU's throttle reasons through NVML at most once a second:
    thermal 3 (hardware thermal slowdown), 2 (software thermal slowdown) or 0."""

    def __init__(self, device_index: Optional[int]):
        self.h = None
        self.last = 0.0
        self.thermal = 0
        if device_index is None:
            return
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(int(device_index))
        except Exception:
            self.h = None

    def poll(self, now: float) -> int:
        if self.h is None or now - self.last < 1.0:
            return self.thermal
        self.last = now
        try:
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            return self.thermal
        self.thermal = 3 if r & 0x40 else (2 if r & 0x20 else 0)
        return self.thermal


class ServingRuntime:
    def __init__(self, pipeline, model_id: str, max_concurrent: int = 4, metrics=None, ctrl: Optional[TPControl] = None,
                 admit_per_step: int = 64):
        self.pipe = pipeline
        self.model_id = model_id
        self.max_concurrent = max_concurrent
        self.metrics = metrics
        self.in_flight = 0
        self._lock = threading.Lock()
        self._pending: "queue.Queue[Submission]" = queue.Queue()
        self._cancel: "queue.Queue[str]" = queue.Queue()
        self._by_id: Dict[str, Submission] = {}
        self._by_rid: Dict[int, Submission] = {}
        self._stop = threading.Event()
        self._wake = threading.Event()
        self.ready = True
        self.broken: Optional[str] = None  # set when a tensor-parallel peer was lost
        self.ctrl = ctrl
        self.engine = getattr(pipeline, "llm", None)
        # admission order: weighted fair queueing over request classes (C++
        # SegmentScheduler), at most `admit_per_step` new requests per engine
        # step, fewer under thermal slowdown
        from .._ext import runtime as _native

        self.admit_per_step = max(1, int(admit_per_step))
        self.segments = _native().SegmentScheduler(self.admit_per_step, True)
        self._held: Dict[str, Submission] = {}
        dev = getattr(getattr(self.engine, "model", None), "device", None)
        self.thermal = ThermalMonitor(getattr(dev, "index", None) if dev is not None else None)
        if ctrl is not None and getattr(ctrl, "heartbeat", None) is None and hasattr(ctrl, "start_heartbeat"):
            ctrl.start_heartbeat(lambda r, why: self._peer_lost(f"tensor-parallel peer lost: {why}"))
        self._thread = threading.Thread(target=self._loop, name="bloom-engine", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------ admission
    def try_acquire(self) -> bool:
        with self._lock:
            if self.in_flight >= self.max_concurrent:
                return False
            self.in_flight += 1
            return True

    def release(self) -> None:
        with self._lock:
            self.in_flight = max(0, self.in_flight - 1)

    @property
    def available_permits(self) -> int:
        return max(0, self.max_concurrent - self.in_flight)

    def submit(self, prompt_ids: List[int], params, messages=None, request_id: Optional[str] = None,
               segment: int = 0) -> Submission:
        loop = asyncio.get_running_loop()
        sub = Submission(request_id or f"req-{next(_ids)}", list(prompt_ids), params, loop, asyncio.Queue(),
                         messages=messages, segment=int(segment))
        if self.broken is not None:
            sub.queue.put_nowait(StreamItem(finished=True, reason="error", error=self.broken))
            return sub
        with self._lock:
            self._by_id[sub.id] = sub
        self._pending.put(sub)
        self._wake.set()
        return sub

    def cancel(self, request_id: str) -> bool:
        with self._lock:
            sub = self._by_id.get(request_id)
        if sub is None:
            return False
        sub.cancelled = True
        self._cancel.put(request_id)
        self._wake.set()
        return True

    def shutdown(self) -> None:
        self._stop.set()
        self._wake.set()
        self._thread.join(timeout=10)
        if self.ctrl is not None and self.engine is not None and self.broken is None:
            self.ctrl.exchange({"stop": True})
        if getattr(self.ctrl, "heartbeat", None) is not None:
            self.ctrl.heartbeat.stop()

    # ------------------------------------------------------------ engine thread
    def _emit(self, sub: Submission, item: StreamItem) -> None:
        sub.loop.call_soon_threadsafe(sub.queue.put_nowait, item)

    def _finish(self, sub: Submission) -> None:
        with self._lock:
            self._by_id.pop(sub.id, None)
            if sub.engine_rid is not None:
                self._by_rid.pop(sub.engine_rid, None)

    def _loop(self) -> None:
        if self.engine is None:
            return self._loop_blocking()
        eng = self.engine
        ctrl = self.ctrl
        last_beat = time.time()
        while not self._stop.is_set():
            msg = {"add": [], "abort": []}
            while True:
                try:
                    rid = self._cancel.get_nowait()
                except queue.Empty:
                    break
                with self._lock:
                    sub = self._by_id.get(rid)
                if sub is not None and sub.engine_rid is not None:
                    eng.abort(sub.engine_rid)
                    msg["abort"].append(sub.engine_rid)
                    self._emit(sub, StreamItem(finished=True, reason="abort"))
                    self._finish(sub)
            while True:
                try:
                    sub = self._pending.get_nowait()
                except queue.Empty:
                    break
                self._held[sub.id] = sub
                self.segments.submit(sub.id, sub.segment)
            if self._held:
                self.segments.set_conditions(self.thermal.poll(time.time()), 0)
            for sid, cls in (self.segments.next_batch() if self._held else []):
                sub = self._held.pop(sid)
                if sub.cancelled:
                    self._emit(sub, StreamItem(finished=True, reason="abort"))
                    self._finish(sub)
                    continue
                prio = SEGMENT_PRIORITY.get(cls, 0)
                try:
                    rid = eng.add_request(sub.prompt_ids, sub.params, prio)
                except Exception as e:  # prompt too long etc.
                    self._emit(sub, StreamItem(finished=True, reason="error", error=str(e)))
                    self._finish(sub)
                    continue
                msg["add"].append((list(sub.prompt_ids), sub.params, prio))
                sub.engine_rid = rid
                with self._lock:
                    self._by_rid[rid] = sub
            msg["step"] = eng.has_unfinished() or bool(self._held)
            if ctrl is not None and (msg["add"] or msg["abort"] or msg["step"] or time.time() - last_beat > 1.0):
                try:
                    ctrl.exchange(msg)  # the other ranks repeat these calls before the same step
                except Exception as e:  # a peer rank is gone (closed connection or process-group timeout)
                    self._peer_lost(f"tensor-parallel peer lost: {e}")
                    return
                last_beat = time.time()
            if not msg["step"]:
                self._wake.wait(timeout=0.05)
                self._wake.clear()
                continue
            if self.broken is not None:  # the heartbeat reported a lost peer
                return
            try:
                outs = eng.step()
                if ctrl is not None and hasattr(ctrl, "tick"):
                    ctrl.tick()
            except Exception as e:  # a failed step fails every request in it (reference mod.rs:1862-1907)
                with self._lock:
                    subs = list(self._by_rid.values())
                for sub in subs:
                    eng.abort(sub.engine_rid)
                    if self.metrics is not None:
                        self.metrics.observe_request(time.time() - sub.created, False, len(sub.prompt_ids))
                    self._emit(sub, StreamItem(finished=True, reason="error", error=f"engine step failed: {e}"))
                    self._finish(sub)
                continue
            now = time.time()
            seen = set()
            for r in outs:  # a request appears once per token of the step (speculation: several)
                if r.request_id in seen:
                    continue
                seen.add(r.request_id)
                sub = self._by_rid.get(r.request_id)
                if sub is None:
                    continue
                if sub.first_token_at is None:
                    sub.first_token_at = now
                    if self.metrics is not None:
                        self.metrics.observe_ttft(now - sub.created)
                new = r.token_ids[sub.n_tokens:]
                if new and self.metrics is not None and sub.last_token_at is not None:
                    self.metrics.observe_itl((now - sub.last_token_at) / len(new))
                if new:
                    sub.last_token_at = now
                if r.finished and self.metrics is not None:
                    self.metrics.observe_request(now - sub.created, r.finish_reason != "error", len(sub.prompt_ids))
                for j, tok in enumerate(new):
                    last = j == len(new) - 1
                    self._emit(sub, StreamItem(token=tok, finished=r.finished and last,
                                               reason=r.finish_reason if last else None))
                sub.n_tokens += len(new)
                if r.finished and not new:  # failed step (kernel status error): no token, an error item
                    self._emit(sub, StreamItem(finished=True, reason=r.finish_reason,
                                               error=getattr(r, "error", None)))
                if r.finished:
                    eng.requests.pop(r.request_id, None)
                    self._finish(sub)

    def _peer_lost(self, reason: str) -> None:
        """No collective can complete any more: every in-flight and queued
        request ends with an error, readiness goes false and new submissions
        are refused with the same reason.  The engine is not stepped again."""
        if self.broken is not None:
            return
        self.broken = reason
        self.ready = False
        with self._lock:
            subs = list(self._by_id.values())
        subs += list(self._held.values())
        self._held.clear()
        while True:
            try:
                subs.append(self._pending.get_nowait())
            except queue.Empty:
                break
        seen = set()
        for sub in subs:
            if sub.id in seen:
                continue
            seen.add(sub.id)
            self._emit(sub, StreamItem(finished=True, reason="error", error=reason))
            self._finish(sub)

    def _loop_blocking(self) -> None:
        """CPU / echo pipelines: one request at a time, text deltas."""
        while not self._stop.is_set():
            try:
                sub = self._pending.get(timeout=0.05)
            except queue.Empty:
                continue
            try:
                reason = "length"
                for delta in self.pipe.run_stream(sub.messages if sub.messages is not None else "", sub.params,
                                                  prompt_ids=sub.prompt_ids if sub.messages is None else None):
                    if sub.cancelled:
                        reason = "abort"
                        break
                    if sub.first_token_at is None:
                        sub.first_token_at = time.time()
                    sub.n_tokens += 1
                    self._emit(sub, StreamItem(text=delta))
                if reason != "abort" and self.pipe.last_generated_tokens < sub.params.max_tokens:
                    reason = "stop"
                self._emit(sub, StreamItem(finished=True, reason=reason))
            except Exception as e:
                self._emit(sub, StreamItem(finished=True, reason="error", error=str(e)))
            self._finish(sub)
