"""Contract tests of the C++ KV block manager and in-flight batching scheduler.

Intent follows the reference's scheduler tests (crates/engine/src/scheduler/
scheduler_test.rs: budgets, decode-before-prefill, chunked prefill splits,
preemption, cancellation, prefix caching and pinning, LRU) with a mock
executor that returns a fixed token, like the reference's MockExecutor.
"""
import pytest
import torch

from bloom_b200._ext import runtime


@pytest.fixture(scope="module")
def rt():
    return runtime()


def make(rt, num_blocks=64, max_seqs=8, budget=64, max_len=512, prefix=True, chunked=True, eos=(2,), buckets=None):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = max_seqs
    cfg.max_num_batched_tokens = budget
    cfg.max_model_len = max_len
    cfg.chunked_prefill = chunked
    cfg.eos_token_ids = list(eos)
    s = rt.Scheduler(cfg, num_blocks, 16, prefix)
    mb = (max_len + 15) // 16
    worst = rt.arena_layout(max(budget, max_seqs), max_seqs, max_seqs, max(budget, max_seqs) // 64 + max_seqs,
                            max(budget, max_seqs) + max_seqs, mb)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, max(budget, max_seqs), max_seqs, mb)
    if buckets:
        s.set_decode_buckets(buckets)
    return s, arena, mb


def params(rt, max_tokens=4, **kw):
    p = rt.SamplingParams()
    p.max_tokens = max_tokens
    p.temperature = 0.0
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def run_step(s, arena, token=42):
    m = s.schedule()
    sampled = torch.full((max(m.num_logits, 1),), token, dtype=torch.int32)
    ev = s.update(sampled, m.num_real_logits)
    return m, ev


def region(arena, off, n, dtype=torch.int32):
    if dtype == torch.int64:
        return arena[off:off + 2 * n].view(torch.int64)
    if dtype == torch.float32:
        return arena[off:off + n].view(torch.float32)
    return arena[off:off + n]


def test_block_manager_prefix_and_lru(rt):
    bm = rt.BlockManager(8, 16, True)
    toks = list(range(40))
    ok, table = bm.allocate([], 40)
    assert ok and len(table) == 3
    hashes = bm.commit(toks, 40, table, [])
    assert len(hashes) == 2  # only full blocks are hashed
    bm.release(table, hashes)
    m = bm.metrics()
    assert m["cached_blocks"] == 2 and m["free_blocks"] == 6
    n, t2, h2 = bm.match_prefix(toks, 39)
    assert n == 32 and t2 == table[:2]
    assert bm.refcount(t2[0]) == 1
    # filling the pool evicts cached blocks only when free ones run out
    ok, t3 = bm.allocate([], 16 * 6)
    assert ok and bm.metrics()["evictions"] == 0
    ok, t4 = bm.allocate([], 16)
    assert not ok  # the two cached blocks are pinned by t2


def test_block_manager_eviction_order(rt):
    bm = rt.BlockManager(4, 16, True)
    a = list(range(32))
    ok, ta = bm.allocate([], 32)
    ha = bm.commit(a, 32, ta, [])
    bm.release(ta, ha)
    ok, tb = bm.allocate([], 48)  # needs one cached block: the tail of prefix a goes first
    assert ok and bm.metrics()["evictions"] == 1
    n, _, _ = bm.match_prefix(a, 31)
    assert n == 16


def test_decode_before_prefill_and_budget(rt):
    s, arena, mb = make(rt, budget=40)
    s.add_request(list(range(10, 40)), params(rt, max_tokens=3))
    m, ev = run_step(s, arena)
    assert m.num_prefill == 1 and m.num_decode == 0 and m.num_tokens == 30 and len(ev) == 1
    s.add_request(list(range(100, 150)), params(rt, max_tokens=3))
    m, ev = run_step(s, arena)
    # decode row of request 1 first, then 39 prefill tokens of request 2 (chunked by the budget)
    assert m.num_decode == 1 and m.num_prefill == 1 and m.num_tokens == 40
    ids = region(arena, m.off_input_ids, m.num_tokens)
    assert int(ids[0]) == 42 and int(ids[1]) == 100
    assert m.num_real_logits == 1  # request 2 not finished prefilling: no sample
    m, ev = run_step(s, arena)
    assert m.num_decode == 1 and m.num_tokens == 1 + 11
    assert m.num_real_logits == 2


def test_positions_slots_and_block_tables(rt):
    s, arena, mb = make(rt, budget=64, prefix=False)
    s.add_request(list(range(3, 23)), params(rt, max_tokens=5))
    m, _ = run_step(s, arena)
    pos = region(arena, m.off_positions, m.num_tokens, torch.int64)
    assert pos.tolist() == list(range(20))
    slots = region(arena, m.off_slot_mapping, m.num_tokens)
    bt = region(arena, m.off_prefill_block_table, mb)
    assert slots.tolist() == [int(bt[p // 16]) * 16 + p % 16 for p in range(20)]
    assert region(arena, m.off_prefill_ctx_lens, 1).tolist() == [20]
    assert region(arena, m.off_prefill_cu_q, 2).tolist() == [0, 20]
    m, _ = run_step(s, arena)
    assert m.num_decode == 1
    assert region(arena, m.off_positions, 1, torch.int64).tolist() == [20]
    assert region(arena, m.off_decode_seq_lens, 1).tolist() == [21]


def test_stop_on_eos_and_max_tokens(rt):
    s, arena, _ = make(rt, eos=(7,))
    r1 = s.add_request([5, 6], params(rt, max_tokens=10))
    r2 = s.add_request([5, 6, 8], params(rt, max_tokens=2, ignore_eos=True))
    m, ev = run_step(s, arena, token=7)
    fin = {e[0]: (e[2], e[3]) for e in ev}
    assert fin[r1] == (True, 1)  # stop (eos)
    assert fin[r2] == (False, 0)
    m, ev = run_step(s, arena, token=9)
    assert ev == [(r2, 9, True, 2)]  # length
    assert not s.has_unfinished()


def test_ignore_eos_and_min_tokens(rt):
    s, arena, _ = make(rt, eos=(7,))
    r = s.add_request([5, 6], params(rt, max_tokens=3, ignore_eos=True))
    for _ in range(2):
        _, ev = run_step(s, arena, token=7)
        assert not ev[0][2]
    _, ev = run_step(s, arena, token=7)
    assert ev[0][2] and ev[0][3] == 2


def test_chunked_prefill_splits(rt):
    s, arena, _ = make(rt, budget=16)
    s.add_request(list(range(50)), params(rt, max_tokens=2))
    lens = []
    for _ in range(4):
        m, ev = run_step(s, arena)
        lens.append(m.num_tokens)
    assert lens == [16, 16, 16, 2 + 1] or lens[:3] == [16, 16, 16]
    assert not s.has_unfinished() or s.num_running == 1


def test_no_chunking_waits_for_budget(rt):
    s, arena, _ = make(rt, budget=32, chunked=False)
    s.add_request(list(range(20)), params(rt))
    s.add_request(list(range(20)), params(rt))
    m, _ = run_step(s, arena)
    assert m.num_prefill == 1 and m.num_tokens == 20


def test_preemption_recompute(rt):
    s, arena, _ = make(rt, num_blocks=4, budget=64, prefix=False, max_seqs=4)
    a = s.add_request(list(range(31)), params(rt, max_tokens=20))
    b = s.add_request(list(range(31)), params(rt, max_tokens=20))
    preempted = 0
    steps = 0
    while s.has_unfinished() and steps < 200:
        m, ev = run_step(s, arena)
        preempted += m.num_preempted
        steps += 1
    assert not s.has_unfinished()
    assert preempted > 0 and s.total_preemptions == preempted


def test_abort(rt):
    s, arena, _ = make(rt)
    a = s.add_request(list(range(20)), params(rt, max_tokens=50))
    run_step(s, arena)
    assert s.abort(a)
    assert not s.abort(a)
    assert not s.has_unfinished()
    assert s.kv_metrics()["active_blocks"] == 0


def test_prefix_reuse_counts(rt):
    s, arena, _ = make(rt, budget=256)
    p = list(range(1000, 1040))
    s.add_request(p, params(rt, max_tokens=1))
    while s.has_unfinished():
        run_step(s, arena)
    r = s.add_request(p + [5, 6], params(rt, max_tokens=1))
    m = s.schedule()
    assert m.num_tokens == 42 - 32  # two cached blocks reused
    assert s.num_cached_prefix(r) == 32
    s.update(torch.zeros(4, dtype=torch.int32), m.num_real_logits)


def test_decode_padding_to_bucket(rt):
    s, arena, mb = make(rt, buckets=[1, 2, 4, 8])
    for i in range(3):
        s.add_request([10 + i, 11, 12], params(rt, max_tokens=4))
    run_step(s, arena)
    m = s.schedule()
    assert m.num_prefill == 0 and m.num_decode == 4 and m.num_real_decode == 3 and m.num_logits == 4
    lay = rt.arena_layout(4, 4, 0, 0, 4, mb)
    assert lay.used_words == m.used_words and lay.off_logits_rows == m.off_logits_rows
    slots = region(arena, m.off_slot_mapping, 4)
    assert int(slots[3]) == -1
    ev = s.update(torch.full((4,), 3, dtype=torch.int32), m.num_real_logits)
    assert len(ev) == 3


def test_priority_order(rt):
    s, arena, _ = make(rt, budget=8, chunked=False)
    lo = s.add_request(list(range(8)), params(rt), priority=0)
    hi = s.add_request(list(range(8)), params(rt), priority=5)
    m, ev = run_step(s, arena)
    assert [e[0] for e in ev] == [hi]


def test_sampling_params_in_arena(rt):
    s, arena, _ = make(rt)
    s.add_request([1, 2, 3], params(rt, temperature=0.5, top_p=0.8, top_k=7, seed=99))
    m = s.schedule()
    assert not m.all_greedy
    assert region(arena, m.off_temperature, 1, torch.float32).tolist() == [0.5]
    assert abs(region(arena, m.off_top_p, 1, torch.float32).item() - 0.8) < 1e-6
    assert region(arena, m.off_top_k, 1).tolist() == [7]
    assert region(arena, m.off_seeds, 1, torch.int64).tolist() == [99]
    s.update(torch.zeros(1, dtype=torch.int32), 1)


def test_many_requests_complete(rt):
    s, arena, _ = make(rt, num_blocks=200, max_seqs=16, budget=128)
    import random

    rng = random.Random(0)
    ids = [s.add_request([rng.randrange(100) for _ in range(rng.randint(1, 90))], params(rt, max_tokens=rng.randint(1, 9)))
           for _ in range(40)]
    done = set()
    for _ in range(2000):
        if not s.has_unfinished():
            break
        m, ev = run_step(s, arena, token=rng.randrange(3, 100))
        for e in ev:
            if e[2]:
                done.add(e[0])
    assert done == set(ids)
    assert s.kv_metrics()["active_blocks"] == 0


def test_cachemesh_offload_restore_and_l3(rt, tmp_path):
    """Evicted prefix blocks go to host slots (L2), spill to files (L3) and come
    back on a later prefix hit; the scheduler queues the copies for the runner."""
    s, arena, mb = make(rt, num_blocks=6, max_seqs=4, budget=64, prefix=True)
    bb = 64
    l2 = torch.zeros(2 * bb, dtype=torch.uint8)  # two host slots
    s.enable_cachemesh(l2, bb, str(tmp_path), 8, "unit")
    import collections

    hbm = collections.defaultdict(lambda: torch.zeros(bb, dtype=torch.uint8))  # simulated device blocks

    def step():
        m = s.schedule()
        for blk, slot in s.take_restores():  # host -> device first
            hbm[blk] = l2[slot * bb:(slot + 1) * bb].clone()
        for blk, slot in s.take_offloads():
            l2[slot * bb:(slot + 1) * bb] = hbm[blk]
        # "forward": every block this step wrote gets a pattern of its first token
        ev = s.update(torch.full((max(m.num_logits, 1),), 7, dtype=torch.int32), m.num_real_logits)
        return m, ev

    def run(prompt):
        rid = s.add_request(prompt, params(rt, max_tokens=1))
        while s.has_unfinished():
            m, _ = step()
        return rid

    a = list(range(100, 133))  # two full blocks + 1
    # device content of A's blocks = a recognisable pattern written at prefill
    s.add_request(a, params(rt, max_tokens=1))
    m = s.schedule()
    assert not s.take_offloads() and not s.take_restores()
    bt = region(arena, m.off_prefill_block_table, mb).tolist()
    for j, blk in enumerate(bt[:3]):
        hbm[blk] = torch.full((bb,), 10 + j, dtype=torch.uint8)
    s.update(torch.full((m.num_logits,), 7, dtype=torch.int32), m.num_real_logits)
    # other prompts evict A's cached blocks (6 HBM blocks in total)
    for base in (200, 300, 400):
        run(list(range(base, base + 33)))
    mm = s.cachemesh_metrics()
    assert mm["offloads"] >= 2 and mm["l3_writes"] >= 1  # 2 host slots: older blocks spilled to files
    # A again: its two full blocks come back from L2 / L3 with their bytes
    s.add_request(a, params(rt, max_tokens=1))
    m = s.schedule()
    rest = s.take_restores()
    assert len(rest) == 2
    for j, (blk, slot) in enumerate(rest):
        assert int(l2[slot * bb]) == 10 + j
    s.take_offloads()
    assert s.cachemesh_metrics()["l2_hits"] + s.cachemesh_metrics()["l3_hits"] == 2


def make_lc(rt, policy, **kw):
    from bloom_b200.engine.engine import apply_long_context_policy

    s, arena, mb = make(rt, **kw)
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = kw.get("max_seqs", 8)
    cfg.max_num_batched_tokens = kw.get("budget", 64)
    cfg.max_model_len = kw.get("max_len", 512)
    cfg.eos_token_ids = [2]
    apply_long_context_policy(cfg, policy)
    s = rt.Scheduler(cfg, kw.get("num_blocks", 64), 16, kw.get("prefix", True))
    s.set_arena(arena, max(cfg.max_num_batched_tokens, cfg.max_num_seqs), cfg.max_num_seqs, mb)
    return s, arena, mb


def test_long_context_visible_blocks(rt):
    # reference paged_cache.rs:1165-1187 with 16-token blocks
    s, _, _ = make_lc(rt, "sliding_window:32")
    assert s.visible_blocks([1, 2, 3, 4]) == [3, 4]
    s, _, _ = make_lc(rt, "context_shift:64:16")
    assert s.visible_blocks([10, 11, 12, 13, 14]) == [12, 13, 14]
    s, _, _ = make_lc(rt, "full")
    assert s.visible_blocks([1, 2, 3]) == [1, 2, 3]
    with pytest.raises(ValueError):
        make_lc(rt, "sliding_window")
    with pytest.raises(ValueError):
        make_lc(rt, "bogus:3")


def test_sliding_window_block_tables(rt):
    s, arena, mb = make_lc(rt, "sliding_window:32", budget=64, prefix=False)
    s.add_request(list(range(3, 103)), params(rt, max_tokens=3))
    m, _ = run_step(s, arena)  # prefill tokens 0..63: the window never starts inside the step
    assert region(arena, m.off_prefill_ctx_lens, 1).tolist() == [64]
    full = region(arena, m.off_prefill_block_table, mb).tolist()
    m, _ = run_step(s, arena)  # tokens 64..99: blocks 4.. visible, context counted from block 4
    assert region(arena, m.off_prefill_ctx_lens, 1).tolist() == [100 - 64]
    bt = region(arena, m.off_prefill_block_table, 3).tolist()
    pos = region(arena, m.off_positions, m.num_tokens, torch.int64).tolist()
    slots = region(arena, m.off_slot_mapping, m.num_tokens).tolist()
    assert pos[0] == 64  # rotary positions and KV slots stay absolute
    assert not set(bt) & set(full[:4])  # the first four blocks are outside the window
    assert all(slots[k] // 16 == bt[p // 16 - 4] for k, p in enumerate(pos))  # table starts at block 4
    table = bt
    m, _ = run_step(s, arena)  # decode at position 100: the last two blocks (32 tokens window)
    assert m.num_decode == 1
    assert region(arena, m.off_decode_seq_lens, 1).tolist() == [101 - 80]
    assert region(arena, m.off_decode_block_table, 2).tolist() == table[1:3]


def test_compact_inactive_releases_cached_blocks(rt):
    s, arena, _ = make_lc(rt, "compact_inactive:8", num_blocks=8, budget=64)
    s.add_request(list(range(500, 540)), params(rt, max_tokens=1))
    while s.has_unfinished():
        run_step(s, arena)
    before = s.kv_metrics()
    assert before["cached_blocks"] >= 2  # full prompt blocks stay in the prefix cache
    assert s.maintain_long_context() == before["cached_blocks"]
    after = s.kv_metrics()
    assert after["free_blocks"] == 8 and after["active_blocks"] == 0


def test_fail_scheduled_frees_kv_and_spares_others(rt):
    """A step whose kernels reported an error: every sequence it scheduled
    finishes with an error and releases its blocks; a waiting request that the
    step did not include is untouched and runs afterwards (reference:
    fail_scheduled_requests, scheduler/mod.rs:1862-1907)."""
    s, arena, _ = make(rt, num_blocks=16, max_seqs=2, budget=64)
    free0 = s.kv_metrics()["free_blocks"]
    a = s.add_request(list(range(3, 40)), params(rt, max_tokens=4))
    b = s.add_request(list(range(5, 30)), params(rt, max_tokens=4))
    c = s.add_request(list(range(7, 20)), params(rt, max_tokens=4))  # max_seqs = 2: waits
    m = s.schedule()
    assert m.num_prefill == 2
    failed = sorted(s.fail_scheduled())
    assert failed == [a, b]
    assert s.kv_metrics()["free_blocks"] == free0
    assert s.num_running == 0 and s.num_waiting == 1
    # the untouched request runs to completion
    done = []
    for _ in range(10):
        if not s.has_unfinished():
            break
        _, ev = run_step(s, arena)
        done += [e for e in ev if e[2]]
    assert [e[0] for e in done] == [c]
    km = s.kv_metrics()  # c's full blocks stay in the prefix cache
    assert km["free_blocks"] + km["cached_blocks"] == free0


# ---------------------------------------------------------------- preemption policies
def _policy_sched(rt, policy, cap=0, priorities=(0, 0, 0, 0), lens=(16, 16, 16, 16), blocks=8):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = 4
    cfg.max_num_batched_tokens = 256
    cfg.max_model_len = 512
    cfg.eos_token_ids = [2]
    cfg.victim_policy = {"newest": 0, "priority": 1, "oldest": 2, "kv_cost": 3, "aegaeon": 4, "lru": 5,
                         "largest_first": 6}[policy]
    cfg.max_preemptions_per_request = cap
    s = rt.Scheduler(cfg, blocks, 16, False)
    mb = 32
    worst = rt.arena_layout(256, 4, 4, 256 // 64 + 4, 256 + 4, mb)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, 256, 4, mb)
    s.set_clock_ms(0.0)
    ids = []
    for i, (p, n) in enumerate(zip(priorities, lens)):
        s.set_clock_ms(float(i) * 1000.0)  # arrivals 1 s apart
        ids.append(s.add_request([3 + i] * n, params(rt, max_tokens=100, ignore_eos=True), p))
    return s, arena, ids


def _victim(rt, s, arena, ids, steps=40):
    for _ in range(steps):
        m = s.schedule()
        sampled = torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32)
        s.update(sampled, m.num_real_logits)
        if m.num_preempted:
            return [i for i in ids if s.num_preemptions(i) > 0]
    return []


def test_victim_policies(rt):
    # 9 blocks of 16 tokens, 4 sequences growing into their 3rd block: one preemption frees enough
    s, arena, ids = _policy_sched(rt, "newest", blocks=9)
    assert _victim(rt, s, arena, ids) == [ids[3]]
    s, arena, ids = _policy_sched(rt, "priority", priorities=(5, 1, 9, 5), blocks=9)
    assert _victim(rt, s, arena, ids) == [ids[1]]  # the lowest priority, even when it is the one asking
    s, arena, ids = _policy_sched(rt, "kv_cost", lens=(20, 18, 17, 24), blocks=9)
    assert _victim(rt, s, arena, ids) == [ids[2]]
    s, arena, ids = _policy_sched(rt, "largest_first", lens=(20, 18, 17, 24), blocks=9)
    assert _victim(rt, s, arena, ids) == [ids[3]]


def test_aegaeon_score_prefers_young_large_sessions(rt):
    """score = age x value / KV tokens: the youngest session holding the most KV goes first."""
    s, arena, ids = _policy_sched(rt, "aegaeon", lens=(17, 17, 17, 30), blocks=9)
    s.set_clock_ms(10_000.0)
    assert _victim(rt, s, arena, ids) == [ids[3]]


def test_preemption_cap_spares_capped_requests(rt):
    """With a cap of 1, a sequence preempted once is only chosen again when no
    other running sequence is left."""
    s, arena, ids = _policy_sched(rt, "newest", cap=1, blocks=9)
    first = _victim(rt, s, arena, ids)
    assert first == [ids[3]]
    for _ in range(200):
        if not s.has_unfinished():
            break
        m = s.schedule()
        sampled = torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32)
        s.update(sampled, m.num_real_logits)
    counts = [s.num_preemptions(i) for i in ids]
    assert all(c in (-1, 0, 1, 2) for c in counts)  # finished ids report -1


def test_kv_admission_threshold_defers_new_requests(rt):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = 8
    cfg.max_num_batched_tokens = 256
    cfg.max_model_len = 512
    cfg.kv_admission_threshold = 0.5
    s = rt.Scheduler(cfg, 8, 16, False)
    worst = rt.arena_layout(256, 8, 8, 256 // 64 + 8, 256 + 8, 32)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, 256, 8, 32)
    a = s.add_request([3] * 70, params(rt, max_tokens=4), 0)  # 5 of 8 blocks
    m = s.schedule()
    s.update(torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32), m.num_real_logits)
    assert s.kv_utilization() >= 0.5
    b = s.add_request([4] * 5, params(rt, max_tokens=4), 0)
    m = s.schedule()
    assert m.num_prefill == 0 and s.num_waiting == 1 and s.admissions_deferred >= 1
    s.update(torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32), m.num_real_logits)
    for _ in range(10):  # a finishes, its blocks free, b is admitted
        if not s.has_unfinished():
            break
        m = s.schedule()
        s.update(torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32), m.num_real_logits)
    assert not s.has_unfinished()


def test_priority_preemption_after_wait_threshold(rt):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = 4
    cfg.max_num_batched_tokens = 256
    cfg.max_model_len = 512
    cfg.priority_preempt_ms = 500.0
    s = rt.Scheduler(cfg, 6, 16, False)
    worst = rt.arena_layout(256, 4, 4, 256 // 64 + 4, 256 + 4, 32)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, 256, 4, 32)
    s.set_clock_ms(0.0)
    low = s.add_request([3] * 90, params(rt, max_tokens=50, ignore_eos=True), 0)  # 6 blocks: the whole pool
    m = s.schedule()
    s.update(torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32), m.num_real_logits)
    high = s.add_request([4] * 20, params(rt, max_tokens=2, ignore_eos=True), 9)
    s.set_clock_ms(100.0)  # waited 100 ms < 500 ms: no preemption yet
    m = s.schedule()
    assert m.num_preempted == 0 and s.num_waiting == 1
    s.update(torch.full((max(m.num_logits, 1),), 42, dtype=torch.int32), m.num_real_logits)
    s.set_clock_ms(700.0)
    m = s.schedule()
    assert m.num_preempted == 1 and s.priority_preemptions == 1
    assert m.num_prefill == 1  # the high-priority request was admitted in the same step
    assert s.num_preemptions(low) == 1 and s.num_waiting == 1


# ---------------------------------------------------------------- swap preemption, state export / import
def _sched(rt, blocks, swap_slots=0, max_seqs=4):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = max_seqs
    cfg.max_num_batched_tokens = 256
    cfg.max_model_len = 512
    cfg.eos_token_ids = [2]
    cfg.swap_slots = swap_slots
    s = rt.Scheduler(cfg, blocks, 16, False)
    worst = rt.arena_layout(256, max_seqs, max_seqs, 256 // 64 + max_seqs, 256 + max_seqs, 32)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, 256, max_seqs, 32)
    return s, arena


def _step(s, tok=42):
    m = s.schedule()
    ev = s.update(torch.full((max(m.num_logits, 1),), tok, dtype=torch.int32), m.num_real_logits)
    return m, ev


def test_swap_preemption_keeps_progress(rt):
    """Swapped-out victims keep their computed tokens: every slot swapped in
    was swapped out before, no prompt token is ever prefilled twice (the
    resumed sequences continue with decode rows), and all slots come back."""
    s, arena = _sched(rt, blocks=9, swap_slots=16)
    ids = [s.add_request([3 + i] * 16, params(rt, max_tokens=40, ignore_eos=True), 0) for i in range(4)]
    held = set()
    prefill_tokens = 0
    swapped_in = 0
    for _ in range(400):
        if not s.has_unfinished():
            break
        m, _ = _step(s)
        prefill_tokens += m.num_tokens - m.num_decode
        for _, slot in s.take_swap_ins():
            assert slot in held
            held.discard(slot)
            swapped_in += 1
        for _, slot in s.take_swap_outs():
            assert slot not in held
            held.add(slot)
    assert not s.has_unfinished()
    assert s.total_swap_outs >= 1 and swapped_in >= 2
    assert prefill_tokens == 4 * 16  # nothing recomputed
    assert not held and s.free_swap_slots == 16


def test_swap_falls_back_to_recompute_without_slots(rt):
    s, arena = _sched(rt, blocks=9, swap_slots=1)  # a victim needs 2 slots
    ids = [s.add_request([3 + i] * 16, params(rt, max_tokens=40, ignore_eos=True), 0) for i in range(4)]
    for _ in range(40):
        _step(s)
        if s.total_preemptions:
            break
    assert s.total_preemptions == 1 and s.total_swap_outs == 0 and not s.take_swap_outs()


def test_export_import_sequence(rt):
    s, arena = _sched(rt, blocks=16)
    a = s.add_request(list(range(3, 40)), params(rt, max_tokens=10, ignore_eos=True), 3)
    for _ in range(3):
        _step(s, 77)
    st = s.export_sequence(a)
    assert st["tokens"][-2:] == [77, 77] and st["num_prompt"] == 37 and st["priority"] == 3
    assert st["num_computed"] == len(st["tokens"]) - 1 and len(st["blocks"]) == (st["num_computed"] + 15) // 16
    free0 = s.kv_metrics()["free_blocks"]
    b, table = s.import_sequence(st["tokens"], st["num_prompt"], st["num_computed"], st["params"], 3)
    assert len(table) == len(st["blocks"]) and not set(table) & set(st["blocks"])
    assert s.kv_metrics()["free_blocks"] == free0 - len(table)
    m, ev = _step(s, 5)
    # the imported sequence needs only its last token computed: a decode row
    assert m.num_prefill == 0 and m.num_decode >= 2
    assert [e[1] for e in ev if e[0] == b] == [5]
    with pytest.raises(Exception):
        s.export_sequence(12345)
    with pytest.raises(Exception):
        s.import_sequence([1] * 600, 1, 10, st["params"], 0)


# ---------------------------------------------------------------- malformed input and overflow safety
# (reference: the scheduler's validation and executor-error tests,
# crates/engine/src/scheduler/scheduler_test.rs:483-613)

def test_invalid_requests_are_refused(rt):
    s, arena, _ = make(rt, num_blocks=8, max_len=128)
    with pytest.raises(ValueError, match="empty prompt"):
        s.add_request([], params(rt))
    with pytest.raises(ValueError, match="max_model_len"):
        s.add_request(list(range(3, 200)), params(rt))
    assert not s.abort(987654)  # unknown ids are not an error
    m = s.schedule()
    assert m.num_tokens == 0 and not s.has_unfinished()


def test_prompt_larger_than_the_pool_is_refused_not_livelocked(rt):
    s, arena, _ = make(rt, num_blocks=4, max_len=512)
    with pytest.raises(ValueError, match="KV blocks"):
        s.add_request(list(range(3, 100)), params(rt))  # 97 tokens > 4 blocks x 16
    assert not s.has_unfinished()


def test_generation_stops_at_pool_capacity(rt):
    s, arena, _ = make(rt, num_blocks=4, max_len=512)
    rid = s.add_request(list(range(3, 40)), params(rt, max_tokens=10_000, ignore_eos=True))
    finished, generated = None, 0
    for _ in range(200):
        _, ev = run_step(s, arena, token=7)
        for r, tok, fin, reason in ev:
            generated += r == rid
            if fin:
                finished = reason
        if not s.has_unfinished():
            break
    assert finished == 2  # length: the pool holds 4 x 16 tokens of one sequence
    assert 37 + generated == 4 * 16
    assert s.kv_metrics()["active_blocks"] == 0


def test_update_rejects_malformed_results(rt):
    s, arena, _ = make(rt)
    s.add_request(list(range(3, 20)), params(rt))
    m = s.schedule()
    with pytest.raises(RuntimeError, match="smaller than n"):
        s.update(torch.zeros(1, dtype=torch.int32), m.num_real_logits + 5)
    with pytest.raises(ValueError, match="fewer sampled tokens"):
        s.update(torch.zeros(4, dtype=torch.int32), 0)
    # the step is still pending: a well-formed result completes it
    ev = s.update(torch.full((max(m.num_logits, 1),), 9, dtype=torch.int32), m.num_real_logits)
    assert len(ev) == 1 and ev[0][1] == 9
