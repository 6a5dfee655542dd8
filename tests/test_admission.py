"""Rate limiter, segment scheduler (WFQ / strict, thermal and power limits) and
the per-device resource ledger (C++), with injected time."""
from bloom_b200._ext import runtime


def test_rate_limiter_buckets():
    rt = runtime()
    off = rt.RateLimiter(False)
    assert off.try_acquire("m", 10 ** 9, 0.0) == (True, 0.0)
    rl = rt.RateLimiter(True, 100.0, 10.0)
    rl.set_override("big", 1000.0, 100.0)
    assert rl.try_acquire("m", 80, 0.0)[0]
    ok, wait = rl.try_acquire("m", 40, 0.0)
    assert not ok and abs(wait - 2.0) < 1e-9  # 20 left, 20 more at 10/s
    assert rl.try_acquire("m", 40, 2.0)[0]
    assert rl.try_acquire("big", 900, 0.0)[0]  # per-model override
    assert abs(rl.available("m", 100.0) - 100.0) < 1e-9  # refills up to the burst only
    assert rl.requests == 4 and rl.throttled == 1


def test_segment_scheduler_wfq_and_limits():
    rt = runtime()
    s = rt.SegmentScheduler(8, True)
    for c in range(4):
        for i in range(10):
            s.submit(f"c{c}-{i}", c)
    b = s.next_batch()
    assert len(b) == 8 and {c for _, c in b} <= {0, 1, 2, 3}
    assert sum(1 for _, c in b if c == 0) >= sum(1 for _, c in b if c == 3)
    strict = rt.SegmentScheduler(5, False)
    for c in (3, 2, 0):
        strict.submit(f"x{c}", c)
    assert [c for _, c in strict.next_batch()] == [0, 2, 3]
    s.set_conditions(2, 0)
    assert s.effective_max_batch() == 4
    s.set_conditions(3, 0)
    assert s.effective_max_batch() == 1 and len(s.next_batch()) == 1
    s.set_conditions(0, 2)
    assert s.effective_max_batch() == 4


def test_resource_ledger_priority_eviction():
    rt = runtime()
    led = rt.ResourceLedger()
    gb = 1 << 30
    led.add_device(0, 180 * gb)
    assert led.reserve("a", 0, 100 * gb, 1, 1) == (True, [])
    assert led.reserve("b", 0, 60 * gb, 2, 2) == (True, [])
    ok, ev = led.reserve("c", 0, 50 * gb, 3, 3)  # evicts the least important (a)
    assert ok and ev == ["a"] and led.free_bytes(0) == 70 * gb
    assert led.reserve("d", 0, 100 * gb, 1, 4) == (False, [])  # nothing less important to evict
    assert led.release("b") and led.used(0) == 50 * gb
