"""int8 paged KV cache on the GPU.

* rope_kv_write into an int8 cache equals the bf16 write quantised per
  (token, head) (values within half a quantisation step);
* decode attention over the int8 cache (int8 Q K^T with per-row quantised
  q, fp16 P V) matches an fp32 softmax over the dequantised pages, including
  split-K and a verify width of 3;
* prefill attention over the int8 cache (dequantised scratch pages) matches
  the fp32 oracle over the same dequantised pages;
* an engine with kv_cache_dtype="int8" generates close to the fp32 oracle
  (the argmax gap criterion of the TP tests, looser for the quantisation).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _caches(nkv, NB=12, seed=0):
    from bloom_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(seed)
    bf = torch.zeros(1, NB, 2, nkv, 16, 128, dtype=torch.bfloat16, device="cuda")
    q8 = torch.zeros(1, NB, ops.kv_q8_block_bytes(nkv), dtype=torch.uint8, device="cuda")
    return g, bf, q8


def test_rope_kv_write_int8_matches_quantised_bf16():
    from bloom_b200 import ops
    from bloom_b200.ops.reference import dequant_q8_cache

    nq, nkv, T = 8, 2, 40
    g, bf, q8 = _caches(nkv)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int64, device="cuda")
    slots = torch.randperm(12 * 16, device="cuda", generator=g)[:T].to(torch.int32)
    cs = ops.rope_cos_sin(256, 128, 10000.0, device="cuda")
    q1 = torch.empty(T, nq, 128, dtype=torch.bfloat16, device="cuda")
    q2 = torch.empty_like(q1)
    ops.rope_kv_write(qkv, pos, slots, cs, q1, bf, 0, nq, nkv)
    ops.rope_kv_write(qkv, pos, slots, cs, q2, q8, 0, nq, nkv)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    deq = dequant_q8_cache(q8, nkv)
    ref = bf.float()
    am = ref.abs().amax(-1, keepdim=True)
    # int8 step (absmax / 254) plus the bf16 rounding of the reference (2^-8 relative)
    excess = (deq - ref).abs() - (am / 254.0 + am * 4e-3 + 1e-6)
    bad = (excess > 0).nonzero()
    assert bad.shape[0] == 0, (bad[:8].tolist(), excess.max().item(), deq[tuple(bad[0].tolist())].item(),
                               ref[tuple(bad[0].tolist())].item(), am[tuple(bad[0].tolist()[:-1] + [0])].item())


@pytest.mark.parametrize("q_len,splits", [(1, 1), (1, 3), (3, 2)])
def test_decode_attention_int8_matches_fp32(q_len, splits):
    from bloom_b200 import ops
    from bloom_b200.ops.reference import dequant_q8_cache

    nq, nkv, NB = 16, 2, 40
    g, bf, q8 = _caches(nkv, NB, seed=q_len * 10 + splits)
    # fill every block through the int8 writer (random K / V rows)
    T = NB * 16
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int64, device="cuda") % 256
    cs = ops.rope_cos_sin(256, 128, 10000.0, device="cuda")
    qo = torch.empty(T, nq, 128, dtype=torch.bfloat16, device="cuda")
    ops.rope_kv_write(qkv, pos, torch.arange(T, dtype=torch.int32, device="cuda"), cs, qo, q8, 0, nq, nkv)
    deq = dequant_q8_cache(q8, nkv)[0]  # [NB, 2, nkv, 16, 128]
    lens = [37, 160, 5, 200]
    B = len(lens)
    perm = torch.randperm(NB, device="cuda", generator=g).to(torch.int32)
    bt = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    for b, L in enumerate(lens):
        n = (L + 15) // 16
        bt[b, :n] = perm[(b * 4) % (NB - n):(b * 4) % (NB - n) + n]
    q = torch.randn(B * q_len, nq, 128, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ops.paged_decode_attention(q, q8, 0, bt, sl, out, q_len=q_len, splits=splits, scale=128 ** -0.5)
    torch.cuda.synchronize()
    assert int(ops.status(0)[0].item()) == 0
    G = nq // nkv
    # the kernel quantises each q row to int8 (absmax / 127) for Q K^T: the
    # same quantisation in the oracle isolates the kernel's arithmetic (tight),
    # exact q bounds the end-to-end error of the int8 path (looser)
    from bloom_b200.ops.reference import quantize_q8_rows

    qi8, qs = quantize_q8_rows(q.float())
    q_deq = qi8 * qs[..., None]
    worst = {"quantised_q": 0.0, "exact_q": 0.0}
    for b, L in enumerate(lens):
        n = (L + 15) // 16
        pages = deq[bt[b, :n].long()]  # [n, 2, nkv, 16, 128]
        k = pages[:, 0].permute(0, 2, 1, 3).reshape(n * 16, nkv, 128)[:L]
        v = pages[:, 1].permute(0, 2, 1, 3).reshape(n * 16, nkv, 128)[:L]
        for qi in range(q_len):
            lim = L - q_len + qi + 1
            for key, qsrc in (("quantised_q", q_deq), ("exact_q", q.float())):
                qq = qsrc[b * q_len + qi].view(nkv, G, 128)
                s = torch.einsum("hgd,khd->hgk", qq, k[:lim]) / math.sqrt(128)
                o = torch.einsum("hgk,khd->hgd", s.softmax(-1), v[:lim]).reshape(nq, 128)
                worst[key] = max(worst[key], (out[b * q_len + qi].float() - o).abs().max().item())
    assert worst["quantised_q"] < 1e-2 and worst["exact_q"] < 4e-2, worst


def test_prefill_attention_int8_matches_fp32():
    from bloom_b200 import ops
    from bloom_b200.ops.reference import attention as ref_attention, dequant_q8_cache

    nq, nkv, NB = 8, 2, 24
    g, bf, q8 = _caches(nkv, NB, seed=5)
    ctx = [70, 33]
    slots, bts = [], []
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(1)).tolist()
    off = 0
    for L in ctx:
        n = (L + 15) // 16
        blocks = perm[off:off + n]
        off += n
        bts.append(blocks + [0] * (8 - n))
        slots += [blocks[t // 16] * 16 + t % 16 for t in range(L)]
    T = sum(ctx)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([t for L in ctx for t in range(L)], dtype=torch.int64, device="cuda")
    cs = ops.rope_cos_sin(256, 128, 10000.0, device="cuda")
    q = torch.empty(T, nq, 128, dtype=torch.bfloat16, device="cuda")
    ops.rope_kv_write(qkv, pos, torch.tensor(slots, dtype=torch.int32, device="cuda"), cs, q, q8, 0, nq, nkv)
    bt = torch.tensor(bts, dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, ctx[0], T], dtype=torch.int32, device="cuda")
    cl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    ts, tst = [t.to("cuda") for t in ops.prefill_tiles([0, ctx[0], T], ctx)]
    out = torch.empty_like(q)
    ops.paged_prefill_attention(q, q8, 0, bt, cl, cu, ts, tst, out, scale=128 ** -0.5)
    torch.cuda.synchronize()
    deq = dequant_q8_cache(q8, nkv)[0]
    worst, a = 0.0, 0
    for s, L in enumerate(ctx):
        n = (L + 15) // 16
        pages = deq[bt[s, :n].long()]
        k = pages[:, 0].permute(0, 2, 1, 3).reshape(n * 16, nkv, 128)[:L]
        v = pages[:, 1].permute(0, 2, 1, 3).reshape(n * 16, nkv, 128)[:L]
        ref = ref_attention(q[a:a + L], k, v, causal=True, scale=128 ** -0.5)
        worst = max(worst, (out[a:a + L].float() - ref).abs().max().item())
        a += L
    assert worst < 2e-2, worst


def test_engine_with_int8_kv_tracks_the_oracle():
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import forward_logits, random_weights

    cfg = preset("tiny-tp")
    w = random_weights(cfg, seed=3, std=0.08, device="cuda")
    model = DecoderLM(cfg, None, "cuda")
    model.shard_full(w)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512, num_blocks=128,
                                        use_cuda_graphs=True, autotune=False, kv_cache_dtype="int8"))
    assert eng.runner.kv_cache.dtype == torch.uint8
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 33, 70, 1)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True))
    worst = 0.0
    for p, o in zip(prompts, outs):
        logits = forward_logits(cfg, w, list(p) + o.token_ids)
        for j, tok in enumerate(o.token_ids):
            row = logits[len(p) - 1 + j]
            spread = (row.max() - row.median()).item()
            worst = max(worst, (row.max() - row[tok]).item() / max(spread, 1e-6))
    assert worst < 0.15, worst
    # export / import keeps the int8 layout
    rid = eng.add_request(prompts[1], SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True))
    eng.step()
    blob = eng.export_state(rid)
    eng.abort(rid)
    rid2 = eng.import_state(blob)
    while eng.has_unfinished():
        eng.step()
    assert len(eng.requests[rid2].token_ids) >= 1
