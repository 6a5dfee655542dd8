"""End-to-end engine on a tiny random model vs the fp32 PyTorch oracle."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
os.environ.setdefault("BLOOM_CHECK_FINITE", "1")


def _build(name, std=0.08, graphs=True, **kw):
    from bloom_b200.engine.engine import EngineConfig, LLMEngine
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset(name)
    w = random_weights(cfg, seed=3, std=std, device="cuda")
    model = DecoderLM(cfg, device="cuda")
    model.shard_full(w)
    ec = EngineConfig(max_num_seqs=kw.get("max_num_seqs", 16), max_num_batched_tokens=kw.get("budget", 512),
                      max_model_len=512, num_blocks=kw.get("num_blocks", 256), use_cuda_graphs=graphs,
                      enable_prefix_caching=kw.get("prefix", True),
                      long_context_policy=kw.get("policy", "full"))
    return cfg, w, LLMEngine(model, ec)


def _check_greedy(cfg, w, prompt, generated):
    from bloom_b200.models.reference import forward_logits

    assert all(0 <= t < cfg.vocab_size for t in generated), generated

    full = list(prompt) + list(generated)
    logits = forward_logits(cfg, w, full)
    for j, tok in enumerate(generated):
        row = logits[len(prompt) - 1 + j]
        spread = (row.max() - row.median()).item()
        gap = (row.max() - row[tok]).item()
        assert gap <= 0.03 * spread + 1e-4, f"step {j}: token {tok} gap {gap} spread {spread}"


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-moe", "tiny-hd64"])
@pytest.mark.parametrize("graphs", [False, True])
def test_engine_greedy_matches_reference(name, graphs):
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, eng = _build(name, graphs=graphs)
    torch.manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,)).tolist() for n in (5, 17, 40, 100, 1)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 12 and o.finished and o.finish_reason == "length"
        _check_greedy(cfg, w, p, o.token_ids)
    from bloom_b200 import ops

    assert int(ops.status()[0].item()) == 0
    if graphs:
        assert eng.runner.stats["graph_steps"] > 0


def test_engine_chunked_prefill_and_prefix_reuse():
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, eng = _build("tiny-llama", budget=48, graphs=False)
    torch.manual_seed(1)
    base = torch.randint(3, cfg.vocab_size, (70,)).tolist()
    outs = eng.generate([base], SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True))
    _check_greedy(cfg, w, base, outs[0].token_ids)
    # same 64-token prefix again: blocks are reused, output unchanged
    m0 = eng.kv_metrics()
    outs2 = eng.generate([base], SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True))
    m1 = eng.kv_metrics()
    assert m1["hits"] > m0["hits"]
    assert outs2[0].token_ids == outs[0].token_ids


def test_engine_preemption_under_kv_pressure():
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, eng = _build("tiny-llama", num_blocks=24, graphs=False, prefix=False)
    torch.manual_seed(2)
    prompts = [torch.randint(3, cfg.vocab_size, (60,)).tolist() for _ in range(6)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=40, temperature=0.0, ignore_eos=True))
    assert eng.scheduler.total_preemptions > 0
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 40
        _check_greedy(cfg, w, p, o.token_ids)


def test_engine_sampling_reproducible():
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, eng = _build("tiny-llama", graphs=True)
    p = [5, 6, 7, 8]
    sp = SamplingParams(max_tokens=10, temperature=0.9, top_p=0.9, seed=1234, ignore_eos=True)
    a = eng.generate([p], sp)[0].token_ids
    b = eng.generate([p], sp)[0].token_ids
    assert a == b and len(a) == 10


def test_engine_json_mode_constrained_decoding():
    import json as _json

    from bloom_b200._ext import runtime
    from bloom_b200.engine.engine import SamplingParams
    from bloom_b200.engine.structured import repair_json
    from bloom_b200.engine.text import Tokenizer

    cfg, w, eng = _build("tiny-llama", graphs=False)
    tok = Tokenizer(None)
    eng.tokenizer = tok
    out = eng.generate([[5, 6, 7]], SamplingParams(max_tokens=24, temperature=0.8, seed=3, json_mode=True,
                                                    ignore_eos=True))[0]
    text = tok.decode(out.token_ids)
    d = runtime().JsonDfa()
    assert d.feed(text), text  # every emitted token kept a valid JSON prefix
    _json.loads(repair_json(text))


def test_moe_routing_kernels_match_reference():
    """Router top-k, grouped expert GEMMs and combine vs the dense fp32 MoE oracle."""
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import moe_mlp, random_weights

    cfg = preset("tiny-moe")
    w = random_weights(cfg, seed=7, std=0.08, device="cuda")
    m = DecoderLM(cfg, device="cuda")
    m.shard_full(w)
    for T in (1, 5, 64, 300, 700):
        x = torch.randn(T, cfg.hidden_size, device="cuda", dtype=torch.bfloat16)
        got = m.moe.forward(0, x)
        exp = moe_mlp(cfg, w, "model.layers.0.", x.float())
        err = ((got.float() - exp).norm() / exp.norm()).item()
        assert err < 2e-2, (T, err)


@pytest.mark.parametrize("E,K,T", [(128, 8, 200), (60, 4, 37), (256, 16, 9)])
def test_moe_route_topk_matches_torch(E, K, T):
    """Register top-k routing: ids, renormalised weights and per-expert slots
    agree with torch.topk of the softmax."""
    from bloom_b200._ext import cuda

    C = cuda()
    g = torch.Generator(device="cuda").manual_seed(E + K + T)
    logits = torch.randn(T, E, device="cuda", generator=g)
    e0, El = E // 4, E // 2
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, K, device="cuda")
    slot = torch.empty(T, K, dtype=torch.int32, device="cuda")
    counts = torch.zeros(El, dtype=torch.int32, device="cuda")
    C.moe_route(logits, K, True, e0, El, ids, wts, slot, counts)
    torch.cuda.synchronize()
    p = logits.softmax(-1)
    tv, ti = p.topk(K, dim=-1)
    assert torch.equal(ids.long(), ti)  # in descending order of probability
    assert torch.allclose(wts, tv / tv.sum(-1, keepdim=True), atol=1e-5)
    loc = (ids >= e0) & (ids < e0 + El)
    assert bool((slot[~loc] == -1).all())
    for e in range(El):
        got = sorted(slot[loc & (ids == e0 + e)].tolist())
        assert got == list(range(int(counts[e]))), (e, got)


@pytest.mark.parametrize("graphs", [False, True])
def test_ngram_speculation_greedy(graphs):
    """n-gram proposals verified in the batched step: greedy outputs still
    follow the oracle, and a repetitive prompt gets proposals accepted."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.engine.speculative import NgramSpeculator
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")
    model = DecoderLM(cfg, device="cuda")
    model.shard_full(w)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512,
                                        num_blocks=256, use_cuda_graphs=graphs, spec_len=4))
    eng.attach_speculator(NgramSpeculator(4, 3))
    torch.manual_seed(5)
    period = torch.randint(3, cfg.vocab_size, (7,)).tolist()
    prompts = [period * 6, torch.randint(3, cfg.vocab_size, (23,)).tolist(), [9]]
    outs = eng.generate(prompts, SamplingParams(max_tokens=20, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 20
        _check_greedy(cfg, w, p, o.token_ids)
    st = eng.speculator.stats(eng)
    assert st["verify_groups"] > 0 and st["proposed"] > 0
    from bloom_b200 import ops

    assert int(ops.status()[0].item()) == 0
    if graphs:
        assert eng.runner.stats["graph_steps"] > 0


def test_draft_model_speculation_same_weights():
    """A draft identical to the target proposes what the target would emit:
    nearly every proposal is accepted and the outputs follow the oracle."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.engine.speculative import DraftModelSpeculator
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")

    def engine(spec_len, mlen, prefix):
        m = DecoderLM(cfg, device="cuda")
        m.shard_full(w)
        return LLMEngine(m, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=mlen,
                                         num_blocks=256, use_cuda_graphs=True, spec_len=spec_len,
                                         enable_prefix_caching=prefix))

    eng = engine(3, 512, True)
    draft = engine(0, 520, False)
    eng.attach_speculator(DraftModelSpeculator(draft, 3))
    torch.manual_seed(6)
    prompts = [torch.randint(3, cfg.vocab_size, (n,)).tolist() for n in (4, 30, 77)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=24, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 24
        _check_greedy(cfg, w, p, o.token_ids)
    st = eng.speculator.stats(eng)
    assert st["acceptance_rate"] > 0.8, st
    assert st["tokens_per_verify"] > 3.0, st


def test_useless_draft_is_paused():
    """A draft with unrelated weights proposes tokens the target rejects: the
    adaptive gate pauses speculation (plain one-row decode steps, captured as
    their own graphs), and the outputs still follow the oracle."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.engine.speculative import DraftModelSpeculator
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")
    wd = random_weights(cfg, seed=99, std=0.08, device="cuda")

    def engine(weights, spec_len, mlen, prefix):
        m = DecoderLM(cfg, device="cuda")
        m.shard_full(weights)
        return LLMEngine(m, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=mlen,
                                         num_blocks=256, use_cuda_graphs=True, spec_len=spec_len,
                                         enable_prefix_caching=prefix, spec_min_acceptance=0.3))

    eng = engine(w, 3, 512, True)
    eng.attach_speculator(DraftModelSpeculator(engine(wd, 0, 520, False), 3))
    torch.manual_seed(7)
    prompts = [torch.randint(3, cfg.vocab_size, (n,)).tolist() for n in (4, 30, 77)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=48, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 48
        _check_greedy(cfg, w, p, o.token_ids)
    st = eng.speculator.stats(eng)
    assert st["gate_pauses"] >= 1, st
    assert st["verify_groups"] < 20, st  # most of the ~48 decode steps ran without a verify width
    assert eng.runner.stats["graph_steps"] > 0


def test_speculation_sampled_runs():
    """Stochastic sampling with proposals: valid tokens, reproducible per seed."""
    from bloom_b200.engine.engine import SamplingParams
    from bloom_b200.engine.speculative import NgramSpeculator

    outs = []
    for _ in range(2):
        from bloom_b200.engine.engine import EngineConfig, LLMEngine
        from bloom_b200.models.config import preset
        from bloom_b200.models.llama import DecoderLM
        from bloom_b200.models.reference import random_weights

        cfg = preset("tiny-llama")
        w = random_weights(cfg, seed=3, std=0.08, device="cuda")
        m = DecoderLM(cfg, device="cuda")
        m.shard_full(w)
        eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                                        num_blocks=128, use_cuda_graphs=False, spec_len=3))
        eng.attach_speculator(NgramSpeculator(3, 2))
        o = eng.generate([[5, 6, 7] * 5], SamplingParams(max_tokens=16, temperature=0.8, top_p=0.95, seed=11,
                                                          ignore_eos=True))
        assert len(o[0].token_ids) == 16 and all(0 <= t < cfg.vocab_size for t in o[0].token_ids)
        outs.append(o[0].token_ids)
    assert outs[0] == outs[1]


def test_cachemesh_restores_evicted_prefix(tmp_path):
    """Prefix blocks evicted from HBM come back from pinned host memory (L2)
    or files (L3) and give the same greedy continuation."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")
    m = DecoderLM(cfg, device="cuda")
    m.shard_full(w)
    from bloom_b200.engine.runner import kv_block_bytes

    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=256, num_blocks=12,
                                    use_cuda_graphs=False, autotune=False,
                                    cachemesh_l2_bytes=3 * kv_block_bytes(m), cachemesh_l3_dir=str(tmp_path),
                                    cachemesh_l3_blocks=64))
    torch.manual_seed(9)
    sp = SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True)
    a = torch.randint(3, cfg.vocab_size, (70,)).tolist()
    first = eng.generate([a], sp)[0].token_ids
    for _ in range(4):  # fill HBM with other prompts: A's cached blocks are evicted
        eng.generate([torch.randint(3, cfg.vocab_size, (70,)).tolist()], sp)
    again = eng.generate([a], sp)[0]
    mesh = eng.kv_metrics()["cachemesh"]
    assert mesh["offloads"] > 0 and mesh["l2_hits"] + mesh["l3_hits"] > 0, mesh
    assert again.token_ids == first
    assert eng.runner.stats["kv_restores"] > 0


@pytest.mark.parametrize("graphs", [False, True])
def test_sliding_window_policy(graphs):
    """A window covering the whole context changes nothing; a 32-token window
    attends to the last two blocks only and still decodes (finite logits,
    no kernel timeouts)."""
    from bloom_b200 import ops
    from bloom_b200.engine.engine import SamplingParams

    torch.manual_seed(1)
    sp = SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True)
    cfg, w, eng = _build("tiny-llama", graphs=graphs, policy="sliding_window:512")
    prompts = [torch.randint(3, cfg.vocab_size, (n,)).tolist() for n in (100, 37, 3)]
    outs = eng.generate(prompts, sp)
    for p, o in zip(prompts, outs):
        _check_greedy(cfg, w, p, o.token_ids)
    _, _, small = _build("tiny-llama", graphs=graphs, policy="sliding_window:32", budget=64)
    outs2 = small.generate(prompts, sp)
    assert all(len(o.token_ids) == 10 and all(0 <= t < cfg.vocab_size for t in o.token_ids) for o in outs2)
    _check_greedy(cfg, w, prompts[2], outs2[2].token_ids)  # 3 + 10 tokens fit in the window
    assert int(ops.status()[0].item()) == 0


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("temperature", [0.0, 0.9])
def test_json_schema_constrained_decoding_random_weights(graphs, temperature):
    """Random weights pick tokens at random; the device vocabulary mask must
    still force every output to be a JSON document the schema accepts,
    ended by end-of-sequence."""
    import json

    from bloom_b200.engine.engine import SamplingParams
    from bloom_b200.engine.structured import validate_json_schema_subset
    from bloom_b200.engine.text import Tokenizer

    cfg, w, eng = _build("tiny-llama", graphs=graphs)
    eng.tokenizer = Tokenizer(None)  # byte tokenizer: ids 3..258 are the bytes, 2 = end of sequence
    schema = {"type": "object", "properties": {"a": {"enum": ["x", "yy"]}, "b": {"type": "boolean"},
                                               "c": {"type": "null"}, "d": {"enum": [1, 22]}},
              "required": ["a", "b", "c", "d"], "additionalProperties": False}
    prompts = [[5, 6, 7], [9, 10, 11, 12, 13], [20] * 30]
    outs = eng.generate(prompts, SamplingParams(max_tokens=250, temperature=temperature, seed=7, json_schema=schema,
                                                stop_token_ids=[2]))
    for o in outs:
        assert o.finish_reason == "stop", (o.finish_reason, o.token_ids)
        body = bytes(t - 3 for t in o.token_ids if 3 <= t < 259).decode()
        assert all(3 <= t < 259 or t == 2 for t in o.token_ids), o.token_ids
        validate_json_schema_subset(json.loads(body), schema)
    from bloom_b200 import ops

    assert int(ops.status()[0].item()) == 0


def test_export_import_state_resumes_identically():
    """Export a running request's KV + tokens, import it into a second engine
    with the same weights: greedy decoding continues with exactly the tokens
    the first engine produces, without recomputing the prefix."""
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, a = _build("tiny-llama", graphs=False)
    _, _, b = _build("tiny-llama", graphs=False)
    sp = SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True)
    prompt = list(range(5, 45))
    rid = a.add_request(prompt, sp)
    for _ in range(6):
        a.step()
    blob = a.export_state(rid)
    got_before = list(a.requests[rid].token_ids)
    while a.has_unfinished():
        a.step()
    full_a = a.requests[rid].token_ids
    rid_b = b.import_state(blob)
    tokens_before = b.runner.stats["tokens"]
    while b.has_unfinished():
        b.step()
    full_b = b.requests[rid_b].token_ids
    assert full_b == full_a, (full_a, full_b)
    assert full_b[:len(got_before)] == got_before
    # only the last token of the imported state was recomputed, then one row per new token
    assert b.runner.stats["tokens"] - tokens_before == 16 - len(got_before)
    _check_greedy(cfg, w, prompt, full_a)
    bad = blob[:12] + blob[12:].replace(b'"head_dim":128', b'"head_dim":64', 1)
    with pytest.raises(ValueError):
        b.import_state(bad)


def test_swap_preemption_matches_reference():
    """A KV pool too small for every request forces preemption; with swap
    space the victims' blocks go to host memory and come back, and greedy
    outputs still match the fp32 oracle."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")
    model = DecoderLM(cfg, device="cuda")
    model.shard_full(w)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512, num_blocks=24,
                                        use_cuda_graphs=True, enable_prefix_caching=False,
                                        swap_space_bytes=64 * 2 * 2 * 2 * 16 * 128 * 2 * 2))
    torch.manual_seed(1)
    prompts = [torch.randint(3, cfg.vocab_size, (40,)).tolist() for _ in range(6)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=40, temperature=0.0, ignore_eos=True))
    assert eng.scheduler.total_swap_outs > 0 and eng.runner.stats.get("swap_ins", 0) > 0
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 40
        _check_greedy(cfg, w, p, o.token_ids)


def test_streamed_layers_match_reference():
    """Layers placed in host memory (streamed into HBM staging slots one layer
    ahead) give the same greedy outputs as the all-HBM model."""
    from bloom_b200.engine.engine import SamplingParams

    cfg, w, eng = _build("tiny-llama", graphs=True)
    m = eng.model
    assert not m.offloaded
    m.place_layers(1)
    assert m.offloaded and m.host_layers == [1] and not m.layers[1]["qkv"].is_cuda
    eng.runner.release_graphs()
    eng.runner.use_cuda_graphs = False
    torch.manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,)).tolist() for n in (5, 40)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        _check_greedy(cfg, w, p, o.token_ids)
