"""Tensor-parallel serving control plane on CPU (gloo, 2 ranks): rank 0's
runtime publishes admissions / aborts / steps, rank 1's follower repeats the
same engine calls in the same order."""
import os
import socket
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = textwrap.dedent(r'''
    import json, os, sys, time, asyncio
    sys.path.insert(0, os.environ["BLOOM_ROOT"])
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="env://")
    from bloom_b200.server.runtime import ServingRuntime, TPControl, follower_loop

    class Out:
        def __init__(self, rid, toks, fin):
            self.request_id, self.token_ids, self.finished, self.finish_reason = rid, toks, fin, "length" if fin else None

    class FakeEngine:
        """Each request gets 3 tokens over 2 steps (2 tokens in its first step: speculation)."""
        def __init__(self):
            self.log, self.next, self.live, self.requests = [], 1, {}, {}
        def add_request(self, prompt, params, priority=0):
            rid = self.next; self.next += 1
            self.live[rid] = []; self.requests[rid] = None
            self.log.append(("add", rid, list(prompt)))
            return rid
        def abort(self, rid):
            self.live.pop(rid, None); self.log.append(("abort", rid))
        def has_unfinished(self):
            return bool(self.live)
        def step(self):
            self.log.append(("step", sorted(self.live)))
            outs = []
            for rid, toks in list(self.live.items()):
                toks.extend([rid * 10 + len(toks), rid * 10 + len(toks) + 1] if not toks else [rid * 10 + len(toks)])
                fin = len(toks) >= 3
                o = Out(rid, list(toks), fin)
                outs += [o] * (2 if len(toks) == 2 else 1)
                if fin:
                    del self.live[rid]
            return outs

    eng = FakeEngine()
    ctrl = TPControl()
    if dist.get_rank() == 0:
        class Pipe: pass
        p = Pipe(); p.llm = eng
        rt = ServingRuntime(p, "fake", 8, ctrl=ctrl)
        async def go():
            subs = [rt.submit([i, i + 1], None) for i in range(3)]
            got = []
            for s in subs:
                toks = []
                while True:
                    it = await s.queue.get()
                    if it.token is not None:
                        toks.append(it.token)
                    if it.finished:
                        break
                got.append(toks)
            return got
        got = asyncio.run(go())
        time.sleep(0.2)
        rt.shutdown()
        print("TOKENS", json.dumps(got))
    else:
        follower_loop(eng, ctrl)
    print("LOG", json.dumps(eng.log))
    dist.barrier()
''')


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_followers_repeat_rank0_calls(tmp_path):
    w = tmp_path / "w.py"
    w.write_text(WORKER)
    port = _port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   BLOOM_ROOT=ROOT)
        procs.append(subprocess.Popen([sys.executable, str(w)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=120) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, o + e
    import json

    logs = [json.loads([l for l in o.splitlines() if l.startswith("LOG")][0][4:]) for o, _ in outs]
    assert logs[0] == logs[1] and any(x[0] == "step" for x in logs[0])
    toks = json.loads([l for l in outs[0][0].splitlines() if l.startswith("TOKENS")][0][7:])
    assert toks == [[10, 11, 12], [20, 21, 22], [30, 31, 32]]  # every token of a multi-token step is delivered


DYING = textwrap.dedent(r'''
    import datetime, json, os, sys, time, asyncio
    sys.path.insert(0, os.environ["BLOOM_ROOT"])
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="env://", timeout=datetime.timedelta(seconds=10))
    from bloom_b200.server.runtime import ServingRuntime, TPControl, follower_loop

    class Out:
        def __init__(self, rid, toks, fin):
            self.request_id, self.token_ids, self.finished, self.finish_reason = rid, toks, fin, "length" if fin else None

    class SlowEngine:
        """Every request needs 1000 steps; rank 1's copy exits after its 3rd step."""
        def __init__(self, die_after=None):
            self.next, self.live, self.requests, self.steps, self.die_after = 1, {}, {}, 0, die_after
        def add_request(self, prompt, params, priority=0):
            rid = self.next; self.next += 1
            self.live[rid] = []; self.requests[rid] = None
            return rid
        def abort(self, rid):
            self.live.pop(rid, None)
        def has_unfinished(self):
            return bool(self.live)
        def step(self):
            self.steps += 1
            outs = []
            for rid, toks in self.live.items():
                toks.append(len(toks))
                outs.append(Out(rid, list(toks), False))
            time.sleep(0.01)
            return outs

    ctrl = TPControl(dist.group.WORLD)
    if dist.get_rank() == 0:
        class Pipe: pass
        p = Pipe(); p.llm = SlowEngine()
        rt = ServingRuntime(p, "fake", 8, ctrl=ctrl)
        async def go():
            subs = [rt.submit([i, i + 1], None) for i in range(2)]
            res = []
            t0 = time.time()
            for s in subs:
                n = 0
                while True:
                    it = await asyncio.wait_for(s.queue.get(), timeout=60)
                    if it.token is not None:
                        n += 1
                    if it.finished:
                        res.append({"tokens": n, "reason": it.reason, "error": it.error})
                        break
            late = rt.submit([9], None)
            it = await asyncio.wait_for(late.queue.get(), timeout=5)
            res.append({"tokens": 0, "reason": it.reason, "error": it.error})
            return res, time.time() - t0
        res, dt = asyncio.run(go())
        print("RESULT", json.dumps({"res": res, "ready": rt.ready, "seconds": dt}), flush=True)
        os._exit(0)
    else:
        eng = SlowEngine()
        orig = eng.step
        def step():
            if eng.steps == 3:
                os._exit(3)  # leaves between steps: after an exchange, before its next step
            return orig()
        eng.step = step
        follower_loop(eng, ctrl)
''')


def test_rank_that_dies_between_steps_fails_requests(tmp_path):
    """Rank 1 exits between two steps.  Rank 0's next lockstep exchange
    raises (closed connection or the 10 s process-group timeout); every
    in-flight request then ends with an error item instead of hanging, the
    runtime reports not-ready and refuses new submissions."""
    import json

    w = tmp_path / "dying.py"
    w.write_text(DYING)
    port = _port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   BLOOM_ROOT=ROOT)
        procs.append(subprocess.Popen([sys.executable, str(w)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=180) for p in procs]
    assert procs[1].returncode == 3, outs[1]
    assert procs[0].returncode == 0, outs[0][0] + outs[0][1]
    line = [l for l in outs[0][0].splitlines() if l.startswith("RESULT")][0]
    r = json.loads(line[7:])
    assert not r["ready"]
    assert len(r["res"]) == 3
    for item in r["res"]:
        assert item["reason"] == "error" and "peer lost" in item["error"], item
    assert r["res"][0]["tokens"] < 1000
