"""Numerics of every sm_100a kernel against plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from bloom_b200 import ops

    return ops


def _ref():
    from bloom_b200.ops import reference

    return reference


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


@pytest.fixture(autouse=True)
def _status_clean():
    ops = _ops()
    ops.status().zero_()
    yield
    torch.cuda.synchronize()
    assert int(ops.status()[0].item()) == 0, "kernel reported a timed-out wait"


@pytest.mark.parametrize("M", [1, 7, 16, 33, 100, 128, 200, 256, 300, 1000])
@pytest.mark.parametrize("N,K", [(128, 64), (384, 256), (1000, 512), (256, 4160)])
def test_gemm_bf16(M, N, K):
    ops, ref = _ops(), _ref()
    torch.manual_seed(M * 7 + N)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    y = ops.gemm(x, w)
    assert rel_err(y, ref.gemm(x, w)) < 1e-2


@pytest.mark.parametrize("M", [5, 64, 257])
def test_gemm_bias_f32_residual(M):
    ops, ref = _ops(), _ref()
    N, K = 512, 384
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    assert rel_err(ops.gemm(x, w, bias=b), ref.gemm(x, w, b)) < 1e-2
    y32 = ops.gemm(x, w, epi=ops.EPI_F32)
    assert y32.dtype == torch.float32 and rel_err(y32, ref.gemm(x, w)) < 1e-3
    r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    yr = ops.gemm(x, w, epi=ops.EPI_RESIDUAL, resid=r)
    assert rel_err(yr, ref.gemm(x, w) + r.float()) < 1e-2


@pytest.mark.parametrize("M,splits", [(3, 2), (64, 4), (256, 3)])
def test_gemm_splitk_partials(M, splits):
    ops, ref = _ops(), _ref()
    N, K = 384, 1024
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    p = ops.gemm(x, w, epi=ops.EPI_PARTIAL_F32, splits=splits)
    assert p.shape == (splits, M, N)
    assert rel_err(p.sum(0), ref.gemm(x, w)) < 1e-3


@pytest.mark.parametrize("M", [1, 40, 256, 700])
def test_gemm_swiglu(M):
    ops, ref = _ops(), _ref()
    I, H = 256, 512
    x = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    g = torch.randn(I, H, device="cuda", dtype=torch.bfloat16) * 0.05
    u = torch.randn(I, H, device="cuda", dtype=torch.bfloat16) * 0.05
    w = ops.interleave_gate_up(g, u)
    y = ops.gemm(x, w, epi=ops.EPI_SWIGLU)
    assert y.shape == (M, I)
    assert rel_err(y, ref.swiglu(ref.gemm(x, g), ref.gemm(x, u))) < 1.5e-2


def test_rmsnorm_and_add():
    ops, ref = _ops(), _ref()
    M, H = 37, 4096
    x = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    assert rel_err(ops.rmsnorm(x, w, 1e-5), ref.rmsnorm(x, w, 1e-5)) < 1e-2
    res = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    d = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    exp_res = (res.float() + d.float())
    r2 = res.clone()
    out = ops.add_rmsnorm(d, r2, w, 1e-5)
    assert rel_err(r2, exp_res) < 1e-2
    assert rel_err(out, ref.rmsnorm(exp_res, w, 1e-5)) < 1.5e-2
    parts = torch.randn(3, M, H, device="cuda", dtype=torch.float32)
    r3 = res.clone()
    out3 = ops.add_rmsnorm(parts, r3, w, 1e-5)
    e3 = res.float() + parts.sum(0)
    assert rel_err(r3, e3) < 1e-2 and rel_err(out3, ref.rmsnorm(e3, w, 1e-5)) < 1.5e-2


def test_layernorm_embedding():
    ops, ref = _ops(), _ref()
    x = torch.randn(10, 384, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(384, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(384, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(10, 384, device="cuda", dtype=torch.bfloat16)
    assert rel_err(ops.layernorm(x, w, b, 1e-12, resid=r), ref.layernorm(x.float() + r.float(), w, b, 1e-12)) < 1e-2
    table = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.tensor([0, 5, 999, 17], device="cuda", dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])


def _make_cache(L, NB, KVH, D=128):
    return torch.randn(L, NB, 2, KVH, 16, D, device="cuda", dtype=torch.bfloat16)


@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("D", [128, 64])
def test_rope_kv_write(qk_norm, D):
    ops, ref = _ops(), _ref()
    T, nq, nkv = 19, 4, 2
    cache = torch.zeros(2, 8, 2, nkv, 16, D, device="cuda", dtype=torch.bfloat16)
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device="cuda", dtype=torch.bfloat16)
    pos = torch.randint(0, 500, (T,), device="cuda", dtype=torch.int64)
    slots = torch.randperm(8 * 16, device="cuda")[:T].to(torch.int32)
    slots[3] = -1
    cs = ops.rope_cos_sin(1024, D, 10000.0, "cuda")
    qn = torch.randn(D, device="cuda", dtype=torch.bfloat16) if qk_norm else None
    kn = torch.randn(D, device="cuda", dtype=torch.bfloat16) if qk_norm else None
    q = torch.empty(T, nq, D, device="cuda", dtype=torch.bfloat16)
    ops.rope_kv_write(qkv, pos, slots, cs, q, cache, 1, nq, nkv, qn, kn, 1e-6)
    v3 = qkv.view(T, nq + 2 * nkv, D).float()
    qr, kr, vr = v3[:, :nq], v3[:, nq:nq + nkv], v3[:, nq + nkv:]
    if qk_norm:
        qr = ref.rmsnorm(qr, qn, 1e-6)
        kr = ref.rmsnorm(kr, kn, 1e-6)
    assert rel_err(q, ref.rope(qr, pos, cs)) < 1e-2
    kexp = ref.rope(kr, pos, cs)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        assert rel_err(cache[1, s // 16, 0, :, s % 16], kexp[t]) < 1e-2
        assert rel_err(cache[1, s // 16, 1, :, s % 16], vr[t]) < 1e-2
    assert cache[0].abs().sum().item() == 0  # other layer untouched


@pytest.mark.parametrize("nq,nkv,q_len", [(32, 8, 1), (8, 8, 1), (16, 2, 1), (32, 8, 4), (8, 1, 4), (8, 1, 5),
                                          (32, 8, 5), (64, 8, 3)])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("D", [128, 64])
def test_paged_decode_attention(nq, nkv, q_len, splits, D):
    ops, ref = _ops(), _ref()
    torch.manual_seed(1)
    L, NB, MB = 2, 300, 64
    cache = _make_cache(L, NB, nkv, D)
    lens = [1, 17, 200, 513, 35, 1000][: 4 if q_len > 1 else 6]
    lens = [max(l, q_len) for l in lens]
    B = len(lens)
    bt = torch.zeros(B, MB, dtype=torch.int32)
    perm = torch.randperm(NB)
    k = 0
    for b, l in enumerate(lens):
        nb = (l + 15) // 16
        bt[b, :nb] = perm[k:k + nb]
        k += nb
    bt = bt.cuda()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B * q_len, nq, D, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    ops.paged_decode_attention(q, cache, 1, bt, sl, out, q_len=q_len, splits=splits, scale=scale)
    for b, l in enumerate(lens):
        kk, vv = ref.gather_paged(cache, 1, bt[b], l)
        exp = ref.attention(q[b * q_len:(b + 1) * q_len], kk, vv, causal=True, q_offset=l - q_len, scale=scale)
        assert rel_err(out[b * q_len:(b + 1) * q_len], exp) < 2e-2, (b, l)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("D", [128, 64])
def test_paged_prefill_attention(causal, D):
    ops, ref = _ops(), _ref()
    torch.manual_seed(2)
    L, NB, MB = 1, 200, 64
    nq, nkv = 8, 2
    cache = _make_cache(L, NB, nkv, D)
    # (prefix already cached, new query tokens)
    seqs = [(0, 5), (0, 64), (32, 100), (16, 1), (100, 250)]
    Sp = len(seqs)
    bt = torch.zeros(Sp, MB, dtype=torch.int32)
    perm = torch.randperm(NB)
    k = 0
    ctx = []
    cu = [0]
    for j, (pre, ql) in enumerate(seqs):
        c = pre + ql
        nb = (c + 15) // 16
        bt[j, :nb] = perm[k:k + nb]
        k += nb
        ctx.append(c)
        cu.append(cu[-1] + ql)
    T = cu[-1]
    q = torch.randn(T, nq, D, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros_like(q)
    tseq, tstart = ops.prefill_tiles(cu, ctx)
    ops.paged_prefill_attention(q, cache, 0, bt.cuda(), torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                                torch.tensor(cu, dtype=torch.int32, device="cuda"), tseq.cuda(), tstart.cuda(), out,
                                scale=1 / math.sqrt(D), causal=causal)
    for j, (pre, ql) in enumerate(seqs):
        kk, vv = ref.gather_paged(cache, 0, bt[j].cuda(), ctx[j])
        exp = ref.attention(q[cu[j]:cu[j + 1]], kk, vv, causal=causal, q_offset=pre, scale=1 / math.sqrt(D))
        assert rel_err(out[cu[j]:cu[j + 1]], exp) < 2e-2, j


def test_argmax_and_sampling():
    ops = _ops()
    B, V = 5, 128256
    logits = torch.randn(B, V, device="cuda", dtype=torch.bfloat16)
    logits[2, 77777] = 50.0
    idx = ops.argmax(logits)
    assert torch.equal(idx.long(), logits.float().argmax(-1))
    temp = torch.tensor([0.0, 1.0, 1.0, 0.7, 1.0], device="cuda")
    top_p = torch.tensor([1.0, 1.0, 0.9, 0.5, 1.0], device="cuda")
    top_k = torch.tensor([0, 1, 0, 0, 3], device="cuda", dtype=torch.int32)
    seeds = torch.arange(B, device="cuda", dtype=torch.int64)
    offs = torch.zeros(B, device="cuda", dtype=torch.int64)
    s = ops.sample(logits, temp, top_p, top_k, seeds, offs)
    assert int(s[0]) == int(idx[0])  # greedy
    assert int(s[1]) == int(idx[1])  # top_k = 1
    assert int(s[2]) == 77777  # overwhelming mass
    third = logits[4].float().topk(3).values[-1].item()
    assert logits[4, int(s[4])].float().item() >= third  # ties with the 3rd value are kept too
    s2 = ops.sample(logits, temp, top_p, top_k, seeds, offs)
    assert torch.equal(s, s2)  # reproducible stream


def test_verify_sampling_is_exact():
    """Rejection sampling against a fixed proposal keeps the target
    distribution: accept d with p(d), else sample p with d removed."""
    ops = _ops()
    V = 48
    probs = torch.softmax(torch.randn(V, device="cuda") * 1.5, 0)
    d = int(probs.argsort()[-3])  # a proposal of middling probability
    n = 40000
    logits = probs.log().unsqueeze(0).repeat(n, 1).contiguous()
    draft = torch.full((n,), d, dtype=torch.int32, device="cuda")
    s = ops.sample(logits, torch.ones(n, device="cuda"), torch.ones(n, device="cuda"),
                   torch.zeros(n, device="cuda", dtype=torch.int32), torch.arange(n, device="cuda"),
                   torch.zeros(n, device="cuda", dtype=torch.int64), draft)
    freq = torch.bincount(s.long(), minlength=V).float() / n
    assert abs(freq[d].item() - probs[d].item()) < 0.015
    assert (freq - probs).abs().max().item() < 0.015
    # greedy rows ignore the proposal and return the argmax
    t0 = torch.zeros(n, device="cuda")
    g = ops.sample(logits[:8], t0[:8], torch.ones(8, device="cuda"), torch.zeros(8, device="cuda", dtype=torch.int32),
                   torch.arange(8, device="cuda"), torch.zeros(8, device="cuda", dtype=torch.int64), draft[:8])
    assert (g.long() == probs.argmax()).all()
    # no proposal (-1) samples as usual; top-p excluding the proposal rejects it surely
    tp = torch.full((n,), 0.3, device="cuda")
    dlow = torch.full((n,), int(probs.argmin()), dtype=torch.int32, device="cuda")
    s3 = ops.sample(logits, torch.ones(n, device="cuda"), tp, torch.zeros(n, device="cuda", dtype=torch.int32),
                    torch.arange(n, device="cuda"), torch.zeros(n, device="cuda", dtype=torch.int64), dlow)
    assert not (s3 == dlow).any()


def test_sampling_distribution():
    ops = _ops()
    V = 64
    probs = torch.softmax(torch.randn(V, device="cuda") * 2, 0)
    logits = probs.log().unsqueeze(0).repeat(4096, 1).contiguous()
    n = logits.shape[0]
    s = ops.sample(logits, torch.ones(n, device="cuda"), torch.ones(n, device="cuda"),
                   torch.zeros(n, device="cuda", dtype=torch.int32), torch.arange(n, device="cuda"),
                   torch.zeros(n, device="cuda", dtype=torch.int64))
    freq = torch.bincount(s.long(), minlength=V).float() / n
    assert (freq - probs).abs().max().item() < 0.03


@pytest.mark.parametrize("M,N,K,splits", [(1, 384, 1024, 3), (64, 4096, 4096, 4), (256, 6144, 4096, 3),
                                          (200, 512, 2048, 5), (512, 1000, 4160, 2)])
@pytest.mark.parametrize("epi", ["bf16", "swiglu", "residual"])
def test_gemm_splitk_fixup(M, N, K, splits, epi):
    ops, ref = _ops(), _ref()
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    if epi == "swiglu":
        N = (N // 32) * 32
        g = torch.randn(N // 2, K, device="cuda", dtype=torch.bfloat16) * 0.05
        u = torch.randn(N // 2, K, device="cuda", dtype=torch.bfloat16) * 0.05
        w = ops.interleave_gate_up(g, u)
        for _ in range(2):  # twice: the per-tile counters must be left at zero
            y = ops.gemm(x, w, epi=ops.EPI_SWIGLU, splits=splits)
            assert rel_err(y, ref.swiglu(ref.gemm(x, g), ref.gemm(x, u))) < 1.5e-2
        return
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    if epi == "bf16":
        for _ in range(2):
            assert rel_err(ops.gemm(x, w, splits=splits), ref.gemm(x, w)) < 1e-2
    else:
        r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
        yr = ops.gemm(x, w, epi=ops.EPI_RESIDUAL, resid=r, splits=splits)
        assert rel_err(yr, ref.gemm(x, w) + r.float()) < 1e-2


@pytest.mark.parametrize("M,N,K,splits", [(64, 1024, 8192, 12), (256, 2048, 8192, 16)])
def test_gemm_splitk_global_fixup(M, N, K, splits):
    """More K-slices than a thread-block cluster holds: the global-memory fixup path."""
    ops, ref = _ops(), _ref()
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    for _ in range(2):
        assert rel_err(ops.gemm(x, w, splits=splits), ref.gemm(x, w)) < 1e-2


@pytest.mark.parametrize("M", [3, 77, 256])
@pytest.mark.parametrize("splits", [1, 3])
def test_gemm_unaligned_output_rows(M, splits):
    """Output rows that are not 16-byte aligned and N not a multiple of 8 take the scalar stores."""
    ops, ref = _ops(), _ref()
    N, K = 100, 1024
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    big = torch.zeros(M, N + 3, device="cuda", dtype=torch.bfloat16)
    out = big[:, 1:N + 1]
    ops.gemm(x, w, out, bias=b if splits == 1 else None, splits=splits)
    want = ref.gemm(x, w, b) if splits == 1 else ref.gemm(x, w)
    assert rel_err(out, want) < 1e-2
    assert big[:, 0].abs().max().item() == 0 and big[:, N + 1:].abs().max().item() == 0
    r = torch.randn(M, N + 5, device="cuda", dtype=torch.bfloat16)[:, 2:N + 2]
    yr = ops.gemm(x, w, epi=ops.EPI_RESIDUAL, resid=r, splits=splits)
    assert rel_err(yr, ref.gemm(x, w) + r.float()) < 1e-2


def test_gemm_auto_splits_decode_shapes():
    ops, ref = _ops(), _ref()
    for M, N, K in [(256, 4096, 14336), (8, 6144, 4096)]:
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        assert rel_err(ops.gemm(x, w), ref.gemm(x, w)) < 1e-2


@pytest.mark.parametrize("kind", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("M", [1, 3, 8, 40])
@pytest.mark.parametrize("epi", ["bf16", "swiglu", "resid"])
def test_gguf_quantized_gemm(kind, M, epi):
    """Block-quantised weights on the GPU vs the fp32 product with the CPU-dequantised weight."""
    from bloom_b200._ext import runtime

    ops, ref = _ops(), _ref()
    torch.manual_seed(0)
    N, K = 512, 1024
    w = torch.randn(N, K) * 0.05
    qw = ops.QWeight.quantize(w, kind, torch.device("cuda"))
    raw = runtime().quantize_q8_0(w.view(-1)) if kind == "Q8_0" else runtime().quantize_q4_0(w.view(-1))
    wd = (runtime().dequant_q8_0(raw, N * K) if kind == "Q8_0" else runtime().dequant_q4_0(raw, N * K)).view(N, K)
    assert torch.equal(qw.dequantize().float().cpu(), wd.to(torch.bfloat16).float())  # bit-exact blocks
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    y = x.float() @ wd.cuda().t()
    if epi == "swiglu":
        out = ops.gemm(x, qw, epi=ops.EPI_SWIGLU)
        g, u = ops.deinterleave_gate_up(wd.cuda())
        exp = torch.nn.functional.silu(x.float() @ g.t()) * (x.float() @ u.t())
    elif epi == "resid":
        r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
        out = ops.gemm(x, qw, epi=ops.EPI_RESIDUAL, resid=r)
        exp = y + r.float()
    else:
        out = ops.gemm(x, qw)
        exp = y
    assert rel_err(out, exp) < 2e-2


def test_gguf_decoder_on_gpu_matches_oracle(tmp_path):
    """A Q8_0 GGUF decoder served from block-quantised GPU weights decodes the
    same greedy tokens as the fp32 oracle on the dequantised weights."""
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.formats.gguf import GGML_Q8_0, GGUFFile, load_hf_weights, write_decoder_gguf
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.reference import forward_logits, random_weights

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=0, std=0.08)
    p = str(tmp_path / "tiny.gguf")
    write_decoder_gguf(p, cfg, w, GGML_Q8_0)
    m = DecoderLM(cfg, device="cuda")
    m.load_gguf(p, quantized=True)
    assert isinstance(m.layers[0]["qkv"], _ops().QWeight)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=256, num_blocks=64,
                                    use_cuda_graphs=True, autotune=False))
    prompts = [[5, 17, 99, 3, 250], [7] * 20]
    outs = eng.generate(prompts, SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True))
    wq = load_hf_weights(GGUFFile(p), dtype=torch.float32)
    for pr, o in zip(prompts, outs):
        logits = forward_logits(cfg, wq, pr + o.token_ids)
        for j, t in enumerate(o.token_ids):
            row = logits[len(pr) - 1 + j]
            assert (row.max() - row[t]).item() <= 0.03 * (row.max() - row.median()).item() + 1e-4


@pytest.mark.parametrize("M,N,K", [(2048, 4096, 4096), (3000, 6272, 1024), (4096, 4736, 2048)])
@pytest.mark.parametrize("epi", ["bf16", "swiglu", "resid"])
def test_gemm_cta_pair_large_m(M, N, K, epi):
    """Large unsplit GEMMs take the 2-CTA (cta_group::2) path: check it
    against fp32, including ragged M / N edges."""
    ops = _ops()
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    if epi == "swiglu":
        N2 = (N // 32) * 32
        w = w[:N2].contiguous()
        out = ops.gemm(x, w, epi=ops.EPI_SWIGLU, splits=1)
        g, u = ops.deinterleave_gate_up(w)
        exp = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    elif epi == "resid":
        r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
        out = ops.gemm(x, w, epi=ops.EPI_RESIDUAL, resid=r, splits=1)
        exp = x.float() @ w.float().t() + r.float()
    else:
        out = ops.gemm(x, w, splits=1)
        exp = x.float() @ w.float().t()
    assert rel_err(out, exp) < 1e-2
    assert int(ops.status()[0].item()) == 0


@pytest.mark.parametrize("M,N,K,bn", [(256, 6144, 4096, 64), (200, 28672, 1024, 32), (96, 8192, 512, 32)])
@pytest.mark.parametrize("epi", ["bf16", "swiglu"])
def test_gemm_cta_pair_small_token_tiles(M, N, K, bn, epi):
    """Decode-sized batches on the CTA-pair kernel with 32 / 64-token tiles."""
    ops = _ops()
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    if epi == "swiglu":
        out = ops.gemm(x, w, epi=ops.EPI_SWIGLU, splits=1, bn=bn)
        g, u = ops.deinterleave_gate_up(w)
        exp = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    else:
        out = ops.gemm(x, w, splits=1, bn=bn)
        exp = x.float() @ w.float().t()
    assert rel_err(out, exp) < 1e-2
    assert int(ops.status()[0].item()) == 0


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_tc_matches_reference_long(causal):
    """tcgen05 prefill attention (S/O in TMEM, lazy rescaling) on long chunks
    with cached prefixes and GQA, against fp32 and the mma.sync kernel."""
    ops, ref = _ops(), _ref()
    torch.manual_seed(5)
    L, NB, D, MB = 1, 600, 128, 160
    nq, nkv = 16, 4
    cache = _make_cache(L, NB, nkv, D)
    seqs = [(0, 700), (1000, 300), (37, 129), (0, 1), (500, 128)]
    bt = torch.zeros(len(seqs), MB, dtype=torch.int32)
    perm = torch.randperm(NB)
    k, ctx, cu = 0, [], [0]
    for j, (pre, ql) in enumerate(seqs):
        c = pre + ql
        nb = (c + 15) // 16
        bt[j, :nb] = perm[k:k + nb]
        k += nb
        ctx.append(c)
        cu.append(cu[-1] + ql)
    q = torch.randn(cu[-1], nq, D, device="cuda", dtype=torch.bfloat16)
    tseq, tstart = ops.prefill_tiles(cu, ctx)
    args = (cache, 0, bt.cuda(), torch.tensor(ctx, dtype=torch.int32, device="cuda"),
            torch.tensor(cu, dtype=torch.int32, device="cuda"), tseq.cuda(), tstart.cuda())
    out_tc = torch.zeros_like(q)
    out_mma = torch.zeros_like(q)
    C = ops._C()
    C.paged_prefill_attention_tc(q, *args, out_tc, 1 / math.sqrt(D), causal, ops.status())
    C.paged_prefill_attention(q, *args, out_mma, 1 / math.sqrt(D), causal, ops.status())
    for j, (pre, ql) in enumerate(seqs):
        kk, vv = ref.gather_paged(cache, 0, bt[j].cuda(), ctx[j])
        exp = ref.attention(q[cu[j]:cu[j + 1]], kk, vv, causal=causal, q_offset=pre, scale=1 / math.sqrt(D))
        assert rel_err(out_tc[cu[j]:cu[j + 1]], exp) < 2e-2, j
        assert rel_err(out_mma[cu[j]:cu[j + 1]], exp) < 2e-2, j
    assert int(ops.status()[0].item()) == 0


# ---------------------------------------------------------------- quantised formats (quant_formats.cu)


def test_int4_flat_dequant_matches_reference():
    ops, ref = _ops(), _ref()
    torch.manual_seed(3)
    n = 128 * 37 + 40
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, ((n + 7) // 8,), dtype=torch.int32)
    sc = torch.rand(n // 128 + 1) + 0.1
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, ((n // 128 + 1 + 7) // 8,), dtype=torch.int32)
    got = ops.dequant_int4_flat(qw.cuda(), sc.cuda(), qz.cuda(), n, dtype=torch.float32).cpu()
    assert torch.allclose(got, ref.dequant_int4_flat(qw, sc, qz, n), atol=1e-5)
    gi = torch.randint(0, sc.numel() + 3, (n - 5,), dtype=torch.int32)  # some groups and ids out of range -> 0
    got = ops.dequant_int4_flat(qw.cuda(), sc.cuda(), qz.cuda(), n, g_idx=gi.cuda(), dtype=torch.float32).cpu()
    assert torch.allclose(got, ref.dequant_int4_flat(qw, sc, qz, n, g_idx=gi), atol=1e-5)


@pytest.mark.parametrize("K,N,G", [(256, 128, 128), (4096, 512, 128), (512, 64, 32)])
def test_gptq_awq_dequant_and_gemm(K, N, G):
    ops, ref = _ops(), _ref()
    torch.manual_seed(K + N)
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32)
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // G, N // 8), dtype=torch.int32)
    sc = (torch.rand(K // G, N) * 0.01 + 0.001).half()
    gi = (torch.arange(K) // G).to(torch.int32)[torch.randperm(K)]  # act-order: permuted groups
    w = ops.dequant_gptq(qw.cuda(), qz.cuda(), sc.cuda(), gi.cuda())
    assert w.shape == (N, K) and rel_err(w.float().cpu(), ref.dequant_gptq(qw, qz, sc, gi)) < 5e-3
    aw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), dtype=torch.int32)
    w2 = ops.dequant_awq(aw.cuda(), qz.cuda(), sc.cuda(), G)
    assert rel_err(w2.float().cpu(), ref.dequant_awq(aw, qz, sc, G)) < 5e-3
    x = torch.randn(33, K, device="cuda", dtype=torch.bfloat16)
    assert rel_err(ops.gemm(x, w2), ref.gemm(x, w2)) < 1e-2


@pytest.mark.parametrize("nf4", [True, False])
def test_bnb4_dequant(nf4):
    ops, ref = _ops(), _ref()
    packed = torch.randint(0, 256, (64 * 100 + 32,), dtype=torch.uint8)
    scale = torch.rand(packed.numel() * 2 // 64 + 1) + 0.5
    got = ops.dequant_bnb4(packed.cuda(), scale.cuda(), 64, nf4=nf4).float().cpu()
    assert rel_err(got, ref.dequant_bnb4(packed, scale, 64, nf4=nf4)) < 5e-3
    g = ops.dequant_bnb4(torch.tensor([23, 240], dtype=torch.uint8, device="cuda"),
                         torch.tensor([2.0], device="cuda"), 4, nf4=nf4).float().cpu()
    want = [-1.3923834, 0.0, 2.0, -2.0] if nf4 else [0.125, 6.0, -6.0, 0.0]
    assert torch.allclose(g, torch.tensor(want), atol=1e-2)


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_kv_row_quant_roundtrip(kind):
    ops, ref = _ops(), _ref()
    x = torch.randn(1000, 1024, device="cuda", dtype=torch.bfloat16)
    x[7] = 0
    q, s = ops.kv_quantize(x, kind)
    y = ops.kv_dequantize(q, s, kind)
    assert s[7].item() == 1.0 and (y[7] == 0).all()
    err = (y.float() - x.float()).abs().max(dim=1).values / x.float().abs().max(dim=1).values.clamp_min(1e-6)
    assert err.max().item() < (0.01 if kind == "int8" else 0.07)
    if kind == "int8":
        qr, sr = ref.kv_quantize_int8(x.float().cpu())
        assert torch.allclose(s.cpu(), sr, rtol=1e-6)
        assert (q.cpu().view(torch.int8).int() - qr.int()).abs().max().item() <= 1


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mrope_cuda_matches_reference(dtype):
    ops, ref = _ops(), _ref()
    torch.manual_seed(2)
    B, H, KVH, S, D = 2, 8, 2, 37, 128
    q = torch.randn(B, H, S, D, device="cuda", dtype=dtype)
    k = torch.randn(B, KVH, S, D, device="cuda", dtype=dtype)
    pos = torch.randint(0, 4096, (3, B, S), device="cuda")
    cos, sin = ops.mrope_cos_sin(pos, D)
    qo, ko = ops.mrope(q, k, cos, sin)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel_err(qo.float().cpu(), ref.mrope(q.float().cpu(), cos.cpu(), sin.cpu())) < tol
    assert rel_err(ko.float().cpu(), ref.mrope(k.float().cpu(), cos.cpu(), sin.cpu())) < tol


@pytest.mark.parametrize("M,splits", [(7, 1), (256, 1), (256, 3), (1000, 1)])
def test_gemm_push_slots(M, splits):
    """Reduce-scatter push addressing, emulated with two local buffers as the
    two ranks' receive buffers: row t lands in buffer t // rows at slot
    [rank][t % rows]; nothing else is written."""
    ops, ref = _ops(), _ref()
    N, K, world, rank = 512, 1024, 2, 1
    rows = (M + world - 1) // world
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    bufs = [torch.zeros(world * rows + 1, N, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ops.gemm(x, w, out, splits=splits, push=([b.data_ptr() for b in bufs], rank, rows))
    want = ref.gemm(x, w)
    for t0 in range(0, M, rows):
        owner = t0 // rows
        got = bufs[owner][rank * rows: rank * rows + min(rows, M - t0)]
        assert rel_err(got, want[t0: t0 + got.shape[0]]) < 1e-2
        assert bufs[owner][: rank * rows].abs().max().item() == 0
        assert bufs[owner][rank * rows + got.shape[0]:].abs().max().item() == 0
