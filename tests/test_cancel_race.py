"""Cancellation against execution in the serving runtime (CPU).

Cancellations arrive from the HTTP side at any time; the runtime applies them
on the engine thread between steps, so an abort never runs while a step is
executing.  Every stream ends exactly once, a cancelled stream ends with
"abort" unless it had already finished, and no token follows the end.
Reference: the execution gate and its tests,
crates/engine/src/scheduler/mod.rs:1458-1460,1526-1532 and
scheduler_test.rs:375-482."""
import asyncio
import random
import threading
import time

from bloom_b200.server.runtime import ServingRuntime


class _Out:
    def __init__(self, rid, toks, fin):
        self.request_id, self.token_ids, self.finished = rid, toks, fin
        self.finish_reason = "length" if fin else None


class _SlowEngine:
    def __init__(self, n_tokens=40):
        self.n_tokens = n_tokens
        self.next, self.live, self.requests = 1, {}, {}
        self.in_step = False
        self.violations = []
        self.aborted = []
        self.lock = threading.Lock()

    def add_request(self, prompt, params, priority=0):
        rid = self.next
        self.next += 1
        self.live[rid] = []
        self.requests[rid] = None
        return rid

    def abort(self, rid):
        if self.in_step:
            self.violations.append(("abort during step", rid))
        self.aborted.append(rid)
        self.live.pop(rid, None)
        return True

    def has_unfinished(self):
        return bool(self.live)

    def step(self):
        self.in_step = True
        try:
            time.sleep(0.002)
            outs = []
            for rid, toks in list(self.live.items()):
                toks.append(rid * 1000 + len(toks))
                fin = len(toks) >= self.n_tokens
                outs.append(_Out(rid, list(toks), fin))
                if fin:
                    del self.live[rid]
            return outs
        finally:
            self.in_step = False


def test_cancellations_never_overlap_a_step_and_every_stream_ends_once():
    eng = _SlowEngine()

    class Pipe:
        llm = eng

    rt = ServingRuntime(Pipe(), "fake", 64)
    rng = random.Random(7)

    async def go():
        subs = [rt.submit([i, i + 1], None) for i in range(24)]
        cancel_at = {s.id: rng.uniform(0.0, 0.12) for s in subs if rng.random() < 0.6}

        async def consume(s):
            toks, ends, after_end = [], [], 0
            while True:
                it = await asyncio.wait_for(s.queue.get(), timeout=20)
                if ends:
                    after_end += 1
                if it.token is not None:
                    toks.append(it.token)
                if it.finished:
                    ends.append(it.reason)
                    # drain anything that would (wrongly) follow the end
                    await asyncio.sleep(0.05)
                    while not s.queue.empty():
                        s.queue.get_nowait()
                        after_end += 1
                    return s.id, toks, ends, after_end

        async def canceller(s, t):
            await asyncio.sleep(t)
            rt.cancel(s.id)

        tasks = [asyncio.create_task(consume(s)) for s in subs]
        cts = [asyncio.create_task(canceller(s, cancel_at[s.id])) for s in subs if s.id in cancel_at]
        res = await asyncio.gather(*tasks)
        await asyncio.gather(*cts)
        return res, cancel_at

    res, cancel_at = asyncio.run(go())
    time.sleep(0.1)
    rt.shutdown()
    assert eng.violations == []
    n_abort = 0
    for sid, toks, ends, after_end in res:
        assert len(ends) == 1 and after_end == 0, (sid, ends, after_end)
        if ends[0] == "abort":
            n_abort += 1
            assert sid in cancel_at
            assert len(toks) < eng.n_tokens
        else:
            assert ends[0] == "length" and len(toks) == eng.n_tokens
        assert toks == sorted(toks)  # in order, no duplicates
        assert len(set(toks)) == len(toks)
    assert n_abort > 0
    assert not eng.live  # nothing left running in the engine
