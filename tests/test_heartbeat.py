"""Store-based liveness of tensor-parallel ranks (CPU, no collective)."""
import multiprocessing as mp
import os
import threading
import time

from bloom_b200.parallel.heartbeat import Heartbeat


class _DictStore:
    def __init__(self):
        self.d = {}

    def set(self, k, v):
        self.d[k] = v.encode() if isinstance(v, str) else v

    def get(self, k):
        return self.d[k]

    def check(self, keys):
        return all(k in self.d for k in keys)


def test_stale_beat_and_step_lag_are_reported_once():
    store = _DictStore()
    lost = []
    h0 = Heartbeat(store, 0, 2, lambda r, why: lost.append((r, why)), stale_s=5.0, max_step_lag=2)
    h1 = Heartbeat(store, 1, 2, lambda r, why: None, stale_s=5.0)
    h0._write()
    h1._write()
    now = time.time()
    h0.check(now)
    assert lost == []
    # rank 1 stops advancing while rank 0 steps on: reported after stale_s of lag
    for _ in range(5):
        h0.tick()
    h1._write()
    h0.check(now)
    h0.check(now + 1.0)
    assert lost == []
    store.set("bloom/hb/1", f"{now + 5.5}:0")  # fresh beat, old step
    h0.check(now + 5.5)
    assert len(lost) == 1 and lost[0][0] == 1 and "stuck" in lost[0][1]
    h0.check(time.time() + 60)
    assert len(lost) == 1  # once


def test_missing_and_old_beats():
    store = _DictStore()
    lost = []
    h0 = Heartbeat(store, 0, 3, lambda r, why: lost.append(r), stale_s=2.0)
    h0._write()
    Heartbeat(store, 1, 3, lambda r, why: None)._write()
    t = time.time()
    h0.check(t)  # rank 2 has not written yet: not lost at once
    assert lost == []
    h0.check(t + 3.0)  # rank 1's beat is 3 s old, rank 2 never wrote
    assert sorted(lost) == [1, 2]


def _child(port, q):
    import torch.distributed as dist

    store = dist.TCPStore("127.0.0.1", port, 2, False, timeout=__import__("datetime").timedelta(seconds=20))
    Heartbeat(store, 1, 2, lambda r, why: None, interval_s=0.2).start()
    q.put("up")
    time.sleep(1.0)
    os._exit(0)  # the rank dies without a word


def test_dead_process_is_detected_through_the_store():
    import datetime

    import torch.distributed as dist

    store = dist.TCPStore("127.0.0.1", 0, 2, True, timeout=datetime.timedelta(seconds=20), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(store.port, q))
    p.start()
    assert q.get(timeout=60) == "up"
    ev = threading.Event()
    why = []
    hb = Heartbeat(store, 0, 2, lambda r, w: (why.append((r, w)), ev.set()), interval_s=0.2, stale_s=1.5).start()
    t0 = time.time()
    assert ev.wait(timeout=20), "the dead rank was not reported"
    assert why[0][0] == 1 and "old" in why[0][1]
    assert time.time() - t0 < 10
    hb.stop()
    p.join(timeout=10)
