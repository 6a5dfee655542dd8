"""Gemma4 kernels and model on the GPU, against plain fp32 PyTorch.

* wide paged decode / verify attention (head_dim 256 and 512, sliding window,
  soft-capped scores, GQA packing, split-K) and chunked-prefill attention;
* the q/k/v norm + partial RoPE + KV page writer (k = v layers included);
* the sandwich residual norm and the GeGLU GEMM epilogue;
* greedy generation through the engine (CUDA graphs, chunked prefill, prompts
  longer than the window) tracks the fp32 Gemma4 oracle.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(NB, nkv, D, E=None, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    E = E or 2 * nkv * 16 * D
    kv = (torch.randn(NB, E, device="cuda", generator=g)).to(torch.bfloat16)
    return kv, g


def _seq_kv(kv, bt_row, L, nkv, D):
    """K, V [L, nkv, D] f32 of one sequence from its pages."""
    n = (L + 15) // 16
    pages = kv[bt_row[:n].long(), :2 * nkv * 16 * D].float().view(n, 2, nkv, 16, D)
    k = pages[:, 0].permute(0, 2, 1, 3).reshape(n * 16, nkv, D)[:L]
    v = pages[:, 1].permute(0, 2, 1, 3).reshape(n * 16, nkv, D)[:L]
    return k, v


def _attend(q, k, v, pos, window, softcap):
    """q [nh, D] at position pos over keys k/v [L, nkv, D] (scale 1)."""
    nh, nkv = q.shape[0], k.shape[1]
    G = nh // nkv
    kk = k.repeat_interleave(G, dim=1)
    vv = v.repeat_interleave(G, dim=1)
    s = torch.einsum("hd,khd->hk", q, kk)
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    j = torch.arange(k.shape[0], device=q.device)
    vis = j <= pos
    if window:
        vis &= j > pos - window
    s = s.masked_fill(~vis[None], float("-inf"))
    return torch.einsum("hk,khd->hd", s.softmax(-1), vv)


@pytest.mark.parametrize("D,nq,nkv,window,softcap,q_len,splits", [
    (256, 8, 4, 40, 50.0, 1, 1),
    (256, 8, 4, 40, 0.0, 3, 4),
    (512, 8, 1, 0, 50.0, 1, 3),
    (512, 16, 1, 0, 0.0, 5, 2),   # 80 packed rows: two row tiles
])
def test_wide_decode_attention(D, nq, nkv, window, softcap, q_len, splits):
    from bloom_b200 import ops

    NB = 48
    E = 2 * nkv * 16 * D + 256  # layer slots wider than this layer needs
    kv, g = _cache(NB, nkv, D, E, seed=D + q_len)
    lens = [37, 160, 5 + q_len, 230]
    B = len(lens)
    perm = torch.randperm(NB, device="cuda", generator=g).to(torch.int32)
    bt = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    for b, L in enumerate(lens):
        n = (L + 15) // 16
        bt[b, :n] = perm[(b * 7) % (NB - n):(b * 7) % (NB - n) + n]
    q = torch.randn(B * q_len, nq, D, device="cuda", generator=g).to(torch.bfloat16) * 0.2
    out = torch.empty_like(q)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = None
    if splits > 1:
        ws = torch.empty(ops.wide_decode_workspace_numel(B, nq, nkv, D, q_len, splits), device="cuda")
    ops.wide_decode_attention(q, kv, nkv, bt, sl, out, q_len=q_len, window=window, softcap=softcap, splits=splits,
                              workspace=ws)
    torch.cuda.synchronize()
    assert int(ops.status(0)[0].item()) == 0
    worst = 0.0
    for b, L in enumerate(lens):
        k, v = _seq_kv(kv, bt[b], L, nkv, D)
        for qi in range(q_len):
            pos = L - q_len + qi
            ref = _attend(q[b * q_len + qi].float(), k, v, pos, window, softcap)
            worst = max(worst, (out[b * q_len + qi].float() - ref).abs().max().item())
    assert worst < 2e-2, worst


@pytest.mark.parametrize("D,nq,nkv,window,softcap", [(256, 4, 2, 24, 30.0), (512, 4, 1, 0, 0.0)])
def test_wide_prefill_attention(D, nq, nkv, window, softcap):
    from bloom_b200 import ops

    NB = 40
    kv, g = _cache(NB, nkv, D, seed=7)
    # (cached prefix, new tokens): a chunk after a prefix, a fresh prompt over two 128-row tiles
    seqs = [(40, 70), (0, 200)]
    bts, ctx, cu = [], [], [0]
    off = 0
    for pre, new in seqs:
        L = pre + new
        n = (L + 15) // 16
        bts.append(list(range(off, off + n)) + [0] * (16 - n))
        off += n
        ctx.append(L)
        cu.append(cu[-1] + new)
    T = cu[-1]
    q = torch.randn(T, nq, D, device="cuda", generator=g).to(torch.bfloat16) * 0.2
    out = torch.empty_like(q)
    bt = torch.tensor(bts, dtype=torch.int32, device="cuda")
    cl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    cuq = torch.tensor(cu, dtype=torch.int32, device="cuda")
    ts, tst = [t.to("cuda") for t in ops.prefill_tiles(cu, ctx)]
    ops.wide_prefill_attention(q, kv, nkv, bt, cl, cuq, ts, tst, out, window=window, softcap=softcap)
    torch.cuda.synchronize()
    assert int(ops.status(0)[0].item()) == 0
    worst = 0.0
    for s, (pre, new) in enumerate(seqs):
        k, v = _seq_kv(kv, bt[s], pre + new, nkv, D)
        for i in range(0, new, 7):
            ref = _attend(q[cu[s] + i].float(), k, v, pre + i, window, softcap)
            worst = max(worst, (out[cu[s] + i].float() - ref).abs().max().item())
    assert worst < 2e-2, worst


@pytest.mark.parametrize("D,rot,k_eq_v", [(256, 256, False), (512, 128, True)])
def test_gemma_qkv_write(D, rot, k_eq_v):
    from bloom_b200 import ops

    nq, nkv, T, NB = 4, 2, 20, 8
    g = torch.Generator(device="cuda").manual_seed(D)
    cols = (nq + nkv * (1 if k_eq_v else 2)) * D
    qkv = torch.randn(T, cols, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 500, (T,), device="cuda", generator=g)
    slots = torch.randperm(NB * 16, device="cuda", generator=g)[:T].to(torch.int32)
    slots[3] = -1  # a padding row writes no KV
    cs = ops.wide_cos_sin(1024, rot, D, 10000.0, "cuda")
    qw = (1 + 0.2 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(D, device="cuda", generator=g)).to(torch.bfloat16)
    E = 2 * nkv * 16 * D
    kv = torch.zeros(NB, E, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(T, nq, D, dtype=torch.bfloat16, device="cuda")
    ops.gemma_qkv_write(qkv, pos, slots, cs, q, kv, nq, nkv, rot, qw, kw, 1e-6, k_eq_v)
    torch.cuda.synchronize()

    def rms(x, w=None):
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
        return y * w.float() if w is not None else y

    def rope(x):
        half = rot // 2
        c = cs[pos][:, None, :half]
        s_ = cs[pos][:, None, half:]
        x1, x2 = x[..., :half], x[..., half:rot]
        return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_, x[..., rot:]], -1)

    f = qkv.float()
    qr = rope(rms(f[:, :nq * D].view(T, nq, D), qw))
    kraw = f[:, nq * D:(nq + nkv) * D].view(T, nkv, D)
    kr = rope(rms(kraw, kw))
    vr = rms(kraw if k_eq_v else f[:, (nq + nkv) * D:].view(T, nkv, D))
    assert (q.float() - qr).abs().max().item() < 3e-2
    pages = kv.float().view(NB, 2, nkv, 16, D)
    for t in range(T):
        sl = int(slots[t])
        if sl < 0:
            continue
        blk, o = sl // 16, sl % 16
        assert (pages[blk, 0, :, o] - kr[t]).abs().max().item() < 3e-2, t
        assert (pages[blk, 1, :, o] - vr[t]).abs().max().item() < 3e-2, t
    # the padding row's would-be slot stays zero
    assert int((pages != 0).any(-1).sum()) == (T - 1) * 2 * nkv


def test_residual_norm_and_softcap():
    from bloom_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(3)
    T, H = 7, 1152
    a = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    x0 = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    wp = (1 + 0.3 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    wn = (1 + 0.3 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()

    x = x0.clone()
    y = ops.residual_norm(a, x, wp, wn, out_scale=0.75)
    torch.cuda.synchronize()
    xr = (x0.float() + rms(a.float(), wp)) * 0.75
    assert (x.float() - xr).abs().max().item() < 2e-2
    assert (y.float() - rms(x.float(), wn)).abs().max().item() < 3e-2
    x2 = torch.empty_like(a)
    y2 = ops.residual_norm(a, x2, None, wn, in_scale=math.sqrt(H))
    torch.cuda.synchronize()
    assert (x2.float() - a.float() * math.sqrt(H)).abs().max().item() < 0.5
    assert (y2.float() - rms(x2.float(), wn)).abs().max().item() < 3e-2
    v = (torch.randn(4, 512, device="cuda", generator=g) * 40).to(torch.bfloat16)
    ref = 30.0 * torch.tanh(v.float() / 30.0)
    ops.softcap_(v, 30.0)
    torch.cuda.synchronize()
    assert (v.float() - ref).abs().max().item() < 0.15


def test_geglu_epilogue():
    from bloom_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(5)
    for M in (3, 200):
        x = torch.randn(M, 256, device="cuda", generator=g).to(torch.bfloat16)
        gate = (torch.randn(512, 256, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        up = (torch.randn(512, 256, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        out = ops.gemm(x, ops.interleave_gate_up(gate, up), epi=ops.EPI_GEGLU)
        torch.cuda.synchronize()
        gt = x.float() @ gate.float().t()
        ref = 0.5 * gt * (1 + torch.tanh(0.7978845608028654 * (gt + 0.044715 * gt ** 3))) * (x.float() @ up.float().t())
        assert out.shape == (M, 512)
        assert (out.float() - ref).abs().max().item() < 3e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("graphs", [False, True])
def test_gemma4_engine_tracks_the_oracle(graphs):
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.gemma4 import Gemma4LM
    from bloom_b200.models.reference import gemma4_forward_logits, gemma4_random_weights

    cfg = preset("tiny-gemma4")
    w = gemma4_random_weights(cfg, seed=2, std=0.08, device="cuda")
    model = Gemma4LM(cfg, None, "cuda")
    model.shard_full(w)
    # a small token budget forces chunked prefill; prompts past the 24-key window
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=64, max_model_len=512,
                                        num_blocks=96, use_cuda_graphs=graphs, autotune=False))
    assert eng.runner.kv_cache.shape == (cfg.num_layers, 96, model.kv_elems)
    gen = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=gen).tolist() for n in (5, 33, 90, 1)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True))
    worst = 0.0
    for p, o in zip(prompts, outs):
        assert len(o.token_ids) == 12
        logits = gemma4_forward_logits(cfg, w, list(p) + o.token_ids)
        for j, tok in enumerate(o.token_ids):
            row = logits[len(p) - 1 + j]
            spread = (row.max() - row.median()).item()
            worst = max(worst, (row.max() - row[tok]).item() / max(spread, 1e-6))
    assert worst < 0.05, worst
