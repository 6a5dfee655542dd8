"""Speculative decoding host logic (CPU): n-gram proposals, verify-group
layout, acceptance / rollback in the C++ scheduler, mirror re-sync, and an
end-to-end check that greedy speculation reproduces plain greedy decoding
with a deterministic mock model (the reference's greedy-equality tests,
crates/engine/src/executor/speculative.rs:891-1271)."""
import pytest
import torch

from bloom_b200._ext import runtime


@pytest.fixture(scope="module")
def rt():
    return runtime()


def make(rt, spec_len, num_blocks=128, max_seqs=8, budget=128, max_len=256, prefix=True, eos=(2,)):
    cfg = rt.SchedulerConfig()
    cfg.max_num_seqs = max_seqs
    cfg.max_num_batched_tokens = budget
    cfg.max_model_len = max_len
    cfg.eos_token_ids = list(eos)
    cfg.spec_len = spec_len
    s = rt.Scheduler(cfg, num_blocks, 16, prefix)
    mb = (max_len + spec_len + 15) // 16
    T = max(budget, max_seqs * (spec_len + 1))
    worst = rt.arena_layout(T, max_seqs, max_seqs, T // 64 + max_seqs, T + max_seqs, mb)
    arena = torch.zeros(worst.used_words, dtype=torch.int32)
    s.set_arena(arena, T, max_seqs, mb)
    return s, arena, mb


def params(rt, max_tokens=16, **kw):
    p = rt.SamplingParams()
    p.max_tokens = max_tokens
    p.temperature = 0.0
    p.ignore_eos = kw.pop("ignore_eos", True)
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def region(arena, off, n, dtype=torch.int32):
    if dtype == torch.int64:
        return arena[off:off + 2 * n].view(torch.int64)
    return arena[off:off + n]


def test_ngram_propose(rt):
    f = rt.ngram_propose
    assert f([1, 2, 3, 4, 1, 2, 3], 3, 4, 1) == [4, 1, 2]
    assert f([5, 6, 7, 5, 6, 9, 5, 6], 2, 4, 1) == [9, 5]  # most recent earlier occurrence wins
    assert f([1, 2, 3], 4, 4, 1) == []
    assert f([7, 7, 7, 7], 2, 2, 1) == [7, 7]
    assert f([1, 2, 3, 9, 1, 2, 3], 6, 4, 2) == [9, 1, 2, 3, 9, 1]  # continues periodically
    assert f([1, 2, 3, 4], 2, 4, 2) == []  # min_order 2: single-token matches ignored


def test_verify_group_layout_and_acceptance(rt):
    s, arena, mb = make(rt, spec_len=3)
    rid = s.add_request(list(range(10, 30)), params(rt))
    m = s.schedule()  # prefill of 20 tokens
    assert m.num_decode == 0 and m.num_prefill == 1 and m.num_logits == 1
    s.update(torch.tensor([100], dtype=torch.int32), 1)
    assert s.decode_candidates() == [rid]
    assert s.set_draft(rid, [101, 102, 103, 999])  # only spec_len proposals are used
    m = s.schedule()
    assert m.num_decode == 1 and m.decode_q_len == 4 and m.num_tokens == 4 and m.num_logits == 4
    assert region(arena, m.off_input_ids, 4).tolist() == [100, 101, 102, 103]
    assert region(arena, m.off_positions, 4, torch.int64).tolist() == [20, 21, 22, 23]
    assert region(arena, m.off_decode_seq_lens, 1).tolist() == [24]
    assert region(arena, m.off_draft_ids, 4).tolist() == [101, 102, 103, -1]
    assert region(arena, m.off_logits_rows, 4).tolist() == [0, 1, 2, 3]
    slots = region(arena, m.off_slot_mapping, 4).tolist()
    assert slots[1] == slots[0] + 1 and len(set(slots)) == 4
    # rows 0, 1 agree with proposals 101, 102; row 2 disagrees -> 55 is the new token
    ev = s.update(torch.tensor([101, 102, 55, 77], dtype=torch.int32), 4)
    assert [e[1] for e in ev] == [101, 102, 55]
    assert s.sequence_tokens(rid)[20:] == [100, 101, 102, 55]
    st = s.spec_stats()
    assert st["verify_groups"] == 1 and st["proposed"] == 3 and st["accepted"] == 2
    # next step starts right after the accepted prefix; with no proposal set
    # on any sequence it is a plain one-row decode (no verify width)
    m = s.schedule()
    assert m.decode_q_len == 1 and m.num_tokens == 1 and m.num_logits == 1
    assert region(arena, m.off_positions, 1, torch.int64).tolist() == [23]
    assert region(arena, m.off_input_ids, 1).tolist() == [55]
    ev = s.update(torch.tensor([60], dtype=torch.int32), 1)
    assert [e[1] for e in ev] == [60]
    # a proposal brings the verify width back
    assert s.set_draft(rid, [61, 62])
    m = s.schedule()
    assert m.decode_q_len == 4 and m.num_tokens == 4
    assert region(arena, m.off_input_ids, 4).tolist() == [60, 61, 62, 0]  # missing proposal: padded
    assert region(arena, m.off_draft_ids, 4).tolist() == [61, 62, -1, -1]


def test_all_accepted_gives_bonus_token(rt):
    s, arena, _ = make(rt, spec_len=2)
    rid = s.add_request([3, 4, 5], params(rt))
    s.schedule()
    s.update(torch.tensor([6], dtype=torch.int32), 1)
    s.set_draft(rid, [7, 8])
    s.schedule()
    ev = s.update(torch.tensor([7, 8, 9], dtype=torch.int32), 3)
    assert [e[1] for e in ev] == [7, 8, 9]
    m = s.schedule()
    assert region(arena, m.off_positions, 1, torch.int64).tolist() == [6]
    assert region(arena, m.off_input_ids, 1).tolist() == [9]


def test_stop_inside_accepted_group(rt):
    s, arena, _ = make(rt, spec_len=3)
    rid = s.add_request([3, 4, 5], params(rt, ignore_eos=False))
    s.schedule()
    s.update(torch.tensor([6], dtype=torch.int32), 1)
    s.set_draft(rid, [7, 2, 8])  # proposal 2 is EOS
    s.schedule()
    ev = s.update(torch.tensor([7, 2, 8, 9], dtype=torch.int32), 4)
    assert [e[1] for e in ev] == [7, 2] and ev[-1][2] and not s.has_unfinished()
    assert s.kv_metrics()["active_blocks"] == 0


def test_max_tokens_cuts_group(rt):
    s, arena, _ = make(rt, spec_len=4)
    rid = s.add_request([3, 4, 5], params(rt, max_tokens=3))
    s.schedule()
    s.update(torch.tensor([6], dtype=torch.int32), 1)
    s.set_draft(rid, [7, 8, 9, 10])
    s.schedule()
    ev = s.update(torch.tensor([7, 8, 9, 10, 11], dtype=torch.int32), 5)
    assert [e[1] for e in ev] == [7, 8] and ev[-1][2] and ev[-1][3] == 2  # length


def test_rejected_rows_free_blocks(rt):
    s, arena, _ = make(rt, spec_len=8, prefix=False)
    rid = s.add_request(list(range(3, 13)), params(rt))  # 10 prompt tokens
    s.schedule()
    s.update(torch.tensor([40], dtype=torch.int32), 1)
    s.set_draft(rid, list(range(41, 49)))
    s.schedule()  # verify rows at positions 10..18 need a second block
    assert s.kv_metrics()["active_blocks"] == 2
    s.update(torch.tensor([1] * 9, dtype=torch.int32), 9)  # nothing accepted
    assert len(s.sequence_tokens(rid)) == 12
    assert s.kv_metrics()["active_blocks"] == 1  # the second block went back to the pool


def test_set_tail_resync(rt):
    s, arena, _ = make(rt, spec_len=0, prefix=False)
    rid = s.add_request([1, 2, 3, 4], params(rt, max_tokens=100))
    for tok in (5, 6, 7):
        s.schedule()
        s.update(torch.tensor([tok], dtype=torch.int32), 1)
    assert s.sequence_tokens(rid) == [1, 2, 3, 4, 5, 6, 7]
    assert s.set_tail(rid, 5, [9, 10])  # keep [1..5], replace the tail
    assert s.sequence_tokens(rid) == [1, 2, 3, 4, 5, 9, 10]
    m = s.schedule()  # 2 tokens to compute again -> a chunk of 2 from position 5
    assert m.num_prefill == 1
    assert region(arena, m.off_positions, 2, torch.int64).tolist() == [5, 6]
    assert not s.set_tail(rid, 2, [])  # cannot cut into the prompt


class MockLM:
    """Deterministic 'model': next token = hash of the last three tokens."""

    V = 11  # a function of the last three tokens over a small alphabet: eventually periodic

    def __call__(self, ctx):
        a, b, c = ([0, 0, 0] + list(ctx))[-3:]
        return (a * 7 + b * 13 + c * 31) % self.V + 3


def drive(rt, spec_len, prompts, max_tokens, proposer):
    """Run the scheduler with a mock executor that evaluates MockLM at every
    sampling row; returns the generated tokens per request."""
    lm = MockLM()
    s, arena, mb = make(rt, spec_len=spec_len, budget=64)
    ids = [s.add_request(p, params(rt, max_tokens=max_tokens)) for p in prompts]
    known = {i: list(p) for i, p in zip(ids, prompts)}
    gen = {i: [] for i in ids}
    steps = 0
    while s.has_unfinished():
        steps += 1
        if spec_len:
            proposer(s, known)
        m = s.schedule()
        rows = s.sampling_ids()
        inp = region(arena, m.off_input_ids, m.num_tokens).tolist()
        lrows = region(arena, m.off_logits_rows, m.num_logits).tolist()
        out = []
        for r, sid in enumerate(rows):
            row = lrows[r]
            if row < m.num_decode * m.decode_q_len:  # verify / decode row
                j = row % m.decode_q_len
                g0 = row - j
                ctx = known[sid] + inp[g0 + 1:g0 + 1 + j]
            else:  # last prompt token of a prefill
                ctx = known[sid]
            out.append(lm(ctx))
        out += [0] * (m.num_logits - len(out))
        ev = s.update(torch.tensor(out or [0], dtype=torch.int32), m.num_real_logits)
        for sid, tok, fin, _ in ev:
            known[sid].append(tok)
            gen[sid].append(tok)
    return [gen[i] for i in ids], steps, s


def test_greedy_speculation_equals_plain_greedy(rt):
    torch.manual_seed(0)
    prompts = [torch.randint(3, 40, (n,)).tolist() for n in (5, 9, 17, 30)]
    plain, plain_steps, _ = drive(rt, 0, prompts, 40, None)

    def ngram(s, known):
        s.propose_ngram(3, 1)

    spec, spec_steps, s = drive(rt, 4, prompts, 40, ngram)
    assert spec == plain
    st = s.spec_stats()
    assert st["accepted"] > 0 and spec_steps < plain_steps  # the mock model is repetitive enough

    lm = MockLM()

    def oracle(s, known):  # perfect proposals: every step accepts all 4 and adds a bonus token
        for sid in s.decode_candidates():
            ctx = list(known[sid])
            d = []
            for _ in range(4):
                d.append(lm(ctx))
                ctx.append(d[-1])
            s.set_draft(sid, d)

    spec2, steps2, _ = drive(rt, 4, prompts, 40, oracle)
    assert spec2 == plain
    assert steps2 <= 1 + (40 + 4) // 5 + 1


class _Sched:
    def __init__(self):
        self.proposed = self.accepted = 0

    def spec_stats(self):
        return {"proposed": self.proposed, "accepted": self.accepted}


def test_adaptive_gate_pauses_and_probes():
    from bloom_b200.engine.speculative import AdaptiveGate

    s = _Sched()
    g = AdaptiveGate(min_acceptance=0.2, alpha=0.5, backoff=4, max_backoff=8)
    assert g.allow(s)  # nothing measured yet
    s.proposed += 16  # a verify step that accepted nothing
    assert not g.allow(s) and g.pauses == 1
    assert [g.allow(s) for _ in range(4)] == [False, False, False, True]  # 4-step pause, then a probe
    s.proposed += 16  # probe also rejected: the pause doubles
    assert not g.allow(s) and g.pauses == 2
    assert sum(1 for _ in range(9) if not g.allow(s)) == 7
    s.proposed += 16
    s.accepted += 12  # the draft became good: proposing continues, backoff resets
    assert g.allow(s) and g.backoff == 4
    assert AdaptiveGate(min_acceptance=0.0).allow(s)  # disabled gate always proposes
