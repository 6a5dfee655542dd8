"""Deterministic record / replay of the scheduler step log (CPU)."""
import json
import random

import torch

from bloom_b200._ext import runtime
from bloom_b200.engine.replay import SchedulerRecorder, replay


def _drive(tmp_path, policy=5, swap_slots=6, seed=0):
    rt = runtime()
    sc = rt.SchedulerConfig()
    sc.max_num_seqs = 6
    sc.max_num_batched_tokens = 64
    sc.max_model_len = 256
    sc.eos_token_ids = [2]
    sc.victim_policy = policy
    sc.priority_preempt_ms = 0.0
    sc.swap_slots = swap_slots
    path = str(tmp_path / "steps.jsonl")
    s = SchedulerRecorder(rt.Scheduler(sc, 14, 16, True), path, sc, 14, 16, True)
    arena = torch.zeros(1 << 16, dtype=torch.int32)
    s.set_arena(arena, 72, 6, 32)
    rng = random.Random(seed)
    ids = []
    for step in range(400):
        if len(ids) < 30 and rng.random() < 0.4:
            sp = rt.SamplingParams()
            sp.max_tokens = rng.randint(1, 30)
            sp.ignore_eos = rng.random() < 0.5
            ids.append(s.add_request([rng.randint(3, 30) for _ in range(rng.randint(1, 90))], sp, rng.randint(0, 3)))
        if ids and rng.random() < 0.05:
            s.abort(rng.choice(ids))
        m = s.schedule()
        s.take_swap_ins()
        s.take_swap_outs()
        if m.num_tokens == 0:
            if len(ids) >= 30 and not s.has_unfinished():
                break
            continue
        if rng.random() < 0.03:
            s.fail_scheduled()
            continue
        sampled = torch.tensor([2 if rng.random() < 0.1 else rng.randint(3, 30)
                                for _ in range(max(1, m.num_logits))], dtype=torch.int32)
        s.update(sampled, m.num_real_logits)
    s.close()
    return path


def test_replay_reproduces_a_recorded_run(tmp_path):
    path = _drive(tmp_path)
    recs = [json.loads(l) for l in open(path)]
    kinds = {r["m"] for r in recs}
    assert {"config", "set_arena", "add", "schedule", "update"} <= kinds
    assert replay(path) is None


def test_replay_reports_the_first_divergence(tmp_path):
    path = _drive(tmp_path, policy=2, swap_slots=0, seed=3)
    lines = open(path).read().splitlines()
    # change the prompt of the third request: its schedule must differ from the log
    n_add = 0
    for i, l in enumerate(lines):
        r = json.loads(l)
        if r["m"] == "add":
            n_add += 1
            if n_add == 3:
                r["prompt"] = [7] * (len(r["prompt"]) + 17)
                lines[i] = json.dumps(r)
                tampered_line = i + 1
                break
    open(path, "w").write("\n".join(lines) + "\n")
    d = replay(path)
    assert d is not None and d["line"] > tampered_line and d["call"] in ("schedule", "update"), d


def test_engine_config_has_step_log():
    from bloom_b200.engine.engine import EngineConfig

    assert EngineConfig().step_log == ""
