"""Per-kernel microbenchmark at the Llama-3-8B serving shapes.

    python -m bloom_b200.cli.kernel_bench [--tp 1] [--json out.json]

Each kernel is timed with CUDA events on the launching stream after warm-up
(median of repeats; operands larger than L2 are rotated between repeats, so
weights and KV pages come from HBM).  Reports achieved TFLOP/s or GB/s and
the fraction of the measured peaks in MEASURED_PEAKS.json (HBM copy
bandwidth, cuBLAS bf16 GEMM), plus torch.matmul (cuBLAS) on the same GEMM
shapes as a library reference point.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch


def load_peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


ITERS = [20]
PROFILE = [False]


def timeit(fn, iters=None, warmup=5):
    """Device time per call: `iters` calls (rotating operands) are captured in
    a CUDA graph and replayed, so host launch cost never shows up in the
    CUDA-event interval; median over 5 replays.  In profile mode (--ncu) the
    op is only launched three times, eagerly, for a profiler to capture."""
    if PROFILE[0]:
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        return float("nan")
    iters = iters or ITERS[0]
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        fn(0)  # allocations of the first call happen outside the capture
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) / iters)
    return statistics.median(ts)


def sweep_gemm(ops, name, M, N, K, epi, x, ws, out, nrot, *, trace, report):
    """Every (token tile, split-K) pair of one GEMM shape: device time per call
    (CUDA graph of back-to-back calls, rotating weights), or with `trace` the
    per-CTA timeline of one launch on a cold weight copy: entry, first stage
    landed, accumulator ready, epilogue done (cluster split-K: slices written),
    cluster barrier passed, reduction + epilogue done; min / median / max in
    microseconds from the first CTA's entry (%globaltimer ticks ~0.26 us)."""
    for bn in (64, 128, 256):
        for sp in (1, 2, 3, 4, 6, 8):
            if K // 64 // sp < 2:
                continue
            extra = {"M": M, "N": N, "K": K, "bn": bn, "splits": sp}
            if trace:
                tr = torch.zeros(8 * 1024, dtype=torch.int64, device=x.device)
                for i in range(3):
                    ops.gemm(x, ws[i % nrot], out, epi=epi, bn=bn, splits=sp)
                torch.cuda.synchronize()
                ops._C().gemm_set_trace(tr)
                ops.gemm(x, ws[3 % nrot], out, epi=epi, bn=bn, splits=sp)
                torch.cuda.synchronize()
                ops._C().gemm_set_trace(None)
                t = tr.view(-1, 8).cpu()
                t = t[t[:, 0] > 0].double()
                if t.shape[0] == 0:  # the 2-CTA kernel ran (it records no timeline)
                    extra["note"] = "2-CTA kernel, no timeline"
                    report(f"gemm_{name}_trace", float("nan"), None, None, extra)
                    continue
                rel = (t - t[:, 0].min()) / 1000.0
                names = {0: "entry", 2: "first_stage", 4: "acc_ready", 5: "written", 7: "cluster_barrier",
                         6: "reduced"}
                for c, nm in names.items():
                    if (t[:, c] > 0).all():
                        extra[nm + "_us"] = [round(float(torch.quantile(rel[:, c], p)), 2) for p in (0.0, 0.5, 1.0)]
                extra["ctas"] = int(t.shape[0])
                report(f"gemm_{name}_trace", float("nan"), None, None, extra)
            else:
                ms = timeit(lambda i=0: ops.gemm(x, ws[i % nrot], out, epi=epi, bn=bn, splits=sp))
                report(f"gemm_{name}_sweep", ms, 2.0 * M * N * K, N * K * 2 + M * K * 2, extra)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--json", default=None)
    ap.add_argument("--only", default="")
    ap.add_argument("--M", type=int, default=0, help="only this token count for GEMMs")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--autotune", action="store_true", help="pick token tile / split-K by measurement first")
    ap.add_argument("--sweep", action="store_true",
                    help="GEMMs: time every (token tile, split-K) pair at the chosen --M instead of the default pick")
    ap.add_argument("--trace", action="store_true",
                    help="GEMMs: per-CTA %%globaltimer phases of one launch per (token tile, split-K) pair")
    ap.add_argument("--ncu", action="store_true",
                    help="profile mode: launch each selected kernel 3 times eagerly, no timing, no cuBLAS runs")
    args = ap.parse_args()
    ITERS[0] = args.iters
    PROFILE[0] = args.ncu
    from bloom_b200 import ops

    hbm, tfl, src = load_peaks()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    t = args.tp
    H, I, V, nq, nkv, hd = 4096, 14336, 128256, 32 // t, max(1, 8 // t), 128
    rows = []

    def report(name, ms, flops=None, bytes_=None, extra=None):
        r = {"kernel": name, "ms": round(ms, 4)}
        if flops:
            r["tflops"] = round(flops / ms / 1e9, 1)
            r["frac_bf16_peak"] = round(flops / ms / 1e9 / tfl, 3)
        if bytes_:
            r["gbs"] = round(bytes_ / ms / 1e6, 1)
            r["frac_hbm_peak"] = round(bytes_ / ms / 1e6 / hbm, 3)
        if extra:
            r.update(extra)
        rows.append(r)
        print(json.dumps(r), flush=True)

    gemms = [("qkv", (nq + 2 * nkv) * hd, H), ("o_proj", H, nq * hd), ("gate_up", 2 * I // t, H),
             ("down", H, I // t), ("lm_head", V // t, H)]
    for M in ((args.M,) if args.M else (1, 64, 256, 2048, 8192)):
        for name, N, K in gemms:
            if args.only and args.only not in ("gemm", name, "gemm_" + name):
                continue
            if name == "lm_head" and M > 256:
                continue
            nrot = max(1, int(math.ceil(400e6 / (N * K * 2))))  # rotate weights beyond L2
            ws = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(nrot)]
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            epi = ops.EPI_SWIGLU if name == "gate_up" else ops.EPI_BF16
            out = torch.empty(M, N // 2 if epi == ops.EPI_SWIGLU else N, device=dev, dtype=torch.bfloat16)
            if args.sweep or args.trace:
                sweep_gemm(ops, name, M, N, K, epi, x, ws, out, nrot, trace=args.trace, report=report)
                del ws
                continue
            if args.autotune and M <= 512:
                ops.gemm_autotune([(N, K, epi == ops.EPI_SWIGLU)], [M], dev)
            ms = timeit(lambda i=0: ops.gemm(x, ws[i % nrot], out, epi=epi))
            flops = 2.0 * M * N * K
            byt = N * K * 2 + M * K * 2 + out.numel() * 2
            extra = {"M": M, "N": N, "K": K}
            tuned = ops.GEMM_TUNED.get((ops._m_bucket(M), N, K, epi == ops.EPI_SWIGLU)) if M <= 512 else None
            if tuned:
                extra["bn_splits"] = list(tuned)
            if M <= 512 and name in ("o_proj", "down") and not args.ncu:
                sp = ops.gemm_default_splits(M, N, K, 0)
                if sp > 1:
                    part = torch.empty(sp, M, N, device=dev, dtype=torch.float32)
                    ms_sk = timeit(lambda i=0: ops.gemm(x, ws[i % nrot], part, epi=ops.EPI_PARTIAL_F32, splits=sp))
                    extra["splitk"] = sp
                    extra["splitk_ms"] = round(ms_sk, 4)
            if not args.ncu:
                cms = timeit(lambda i=0: torch.matmul(x, ws[i % nrot].t()))
                extra["cublas_ms"] = round(cms, 4)
            report(f"gemm_{name}", ms, flops, byt, extra)
            del ws

    if not args.only or "attn" in args.only or "attention" in args.only:
        # decode attention: 256 sequences, context U[512, 2304]
        import random

        rng = random.Random(0)
        B = 256
        lens = [rng.randint(512, 2304) for _ in range(B)]
        MB = 2304 // 16
        NB = sum((l + 15) // 16 for l in lens) + 8
        L = 2
        cache = torch.randn(L, NB, 2, nkv, 16, hd, device=dev, dtype=torch.bfloat16)
        bt = torch.zeros(B, MB, dtype=torch.int32)
        perm = torch.randperm(NB)
        k = 0
        for b, l in enumerate(lens):
            nb = (l + 15) // 16
            bt[b, :nb] = perm[k:k + nb]
            k += nb
        bt = bt.to(dev)
        sl = torch.tensor(lens, dtype=torch.int32, device=dev)
        q = torch.randn(B, nq, hd, device=dev, dtype=torch.bfloat16)
        o = torch.empty_like(q)
        splits = ops.decode_attention_splits(B, nkv, MB, 0)
        ws = torch.empty(ops.decode_workspace_numel(B, nkv, splits), device=dev)
        kv_bytes = sum(lens) * nkv * hd * 2 * 2
        ms = timeit(lambda i=0: ops.paged_decode_attention(q, cache, i % L, bt, sl, o, splits=splits, workspace=ws,
                                                           scale=hd ** -0.5))
        report("paged_decode_attention", ms, None, kv_bytes, {"B": B, "avg_ctx": sum(lens) / B, "splits": splits})
        if hd == 128:
            # the same workload over an int8 cache (1 byte per element + 4 bytes of scale per token and head)
            cache8 = torch.randint(0, 256, (L, NB, ops.kv_q8_block_bytes(nkv)), dtype=torch.uint8, device=dev)
            sc_off = 2 * nkv * 16 * hd
            cache8[:, :, sc_off:] = torch.full((L, NB, 2 * nkv * 16), 0.01, device=dev).view(torch.uint8).view(
                L, NB, -1)
            ms8 = timeit(lambda i=0: ops.paged_decode_attention(q, cache8, i % L, bt, sl, o, splits=splits,
                                                                workspace=ws, scale=hd ** -0.5))
            report("paged_decode_attention_int8", ms8, None, sum(lens) * nkv * (hd + 4) * 2,
                   {"B": B, "avg_ctx": sum(lens) / B, "splits": splits, "speedup_vs_bf16": round(ms / ms8, 2)})
            del cache8
        for Bs in (() if args.ncu else (1, 8, 32)):
            sl2 = sl[:Bs].contiguous()
            sp = ops.decode_attention_splits(Bs, nkv, MB, 0)
            ws2 = torch.empty(ops.decode_workspace_numel(Bs, nkv, sp), device=dev)
            ms = timeit(lambda i=0: ops.paged_decode_attention(q[:Bs], cache, i % L, bt[:Bs], sl2, o[:Bs], splits=sp,
                                                               workspace=ws2, scale=hd ** -0.5))
            report(f"paged_decode_attention_b{Bs}", ms, None, sum(lens[:Bs]) * nkv * hd * 4,
                   {"B": Bs, "splits": sp})
        # prefill attention: 4 sequences x 2048 tokens, causal
        S, Lq = 4, 2048
        NB2 = S * Lq // 16
        cache2 = torch.randn(1, NB2, 2, nkv, 16, hd, device=dev, dtype=torch.bfloat16)
        bt2 = torch.arange(NB2, dtype=torch.int32, device=dev).view(S, Lq // 16).contiguous()
        cu = [i * Lq for i in range(S + 1)]
        ctx = [Lq] * S
        tseq, tstart = ops.prefill_tiles(cu, ctx)
        q2 = torch.randn(S * Lq, nq, hd, device=dev, dtype=torch.bfloat16)
        o2 = torch.empty_like(q2)
        ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        ts_, tst = tseq.to(dev), tstart.to(dev)
        ms = timeit(lambda i=0: ops.paged_prefill_attention(q2, cache2, 0, bt2, ctx_t, cu_t, ts_, tst, o2,
                                                            scale=hd ** -0.5))
        flops = S * 4.0 * Lq * Lq / 2 * hd * nq
        report("paged_prefill_attention", ms, flops, None, {"seqs": S, "len": Lq})
        if args.trace:
            # per-CTA phase profile of one launch: thread 0's clock64 cycles per kv tile
            ctas = int(ts_.numel()) * nq
            tr = torch.zeros(ctas * 16, dtype=torch.int64, device=dev)
            ops._C().attn_tc_set_trace(tr)
            ops.paged_prefill_attention(q2, cache2, 0, bt2, ctx_t, cu_t, ts_, tst, o2, scale=hd ** -0.5)
            torch.cuda.synchronize()
            ops._C().attn_tc_set_trace(None)
            t = tr.view(ctas, 16).cpu().double()
            t = t[t[:, 0] > 0]
            nkt = t[:, 10].sum().item()
            names = ["issue_S_next", "barrier", "wait_S", "load_S_rowmax", "wait_PV_prev", "exp_P_store",
                     "issue_PV"]
            extra = {"ctas": int(t.shape[0]), "kv_tiles": int(nkt),
                     "loop_cycles_per_tile": round(t[:, 2].sum().item() / max(nkt, 1), 1),
                     "launch_us": round((t[:, 1].max() - t[:, 0].min()).item() / 1000.0, 2),
                     "cta_us_median": round(float((t[:, 1] - t[:, 0]).median()) / 1000.0, 2)}
            for k, nm in enumerate(names):
                extra[nm + "_cycles_per_tile"] = round(t[:, 3 + k].sum().item() / max(nkt, 1), 1)
            extra["mma_warp_wait_K_cycles_per_tile"] = round(t[:, 11].sum().item() / max(nkt, 1), 1)
            extra["mma_warp_wait_V_cycles_per_tile"] = round(t[:, 12].sum().item() / max(nkt, 1), 1)
            extra["mma_warp_wait_QP_cycles_per_tile"] = round(t[:, 13].sum().item() / max(nkt, 1), 1)
            extra["mma_warp_wait_Sfree_cycles_per_tile"] = round(t[:, 14].sum().item() / max(nkt, 1), 1)
            report("paged_prefill_attention_profile", float("nan"), None, None, extra)

    if not args.only or "gemma" in args.only:
        # Gemma4 wide-head attention, 64 sequences of 4,096 tokens: sliding layer (head_dim 256,
        # 16 q / 8 KV heads, 1,024-key window, soft-cap 50) and global layer (head_dim 512, 16 q / 1
        # KV head), decode and a 2 x 2,048-token prefill chunk; bytes = the KV pages a step must read
        for D, gnq, gkv, win in ((256, 16, 8, 1024), (512, 16, 1, 0)):
            B, ctx = 64, 4096
            MB = ctx // 16
            E = 2 * gkv * 16 * D
            NB = B * MB
            kvl = torch.randn(NB, E, device=dev, dtype=torch.bfloat16)
            bt = torch.randperm(NB, device=dev).to(torch.int32).view(B, MB)
            sl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
            q = torch.randn(B, gnq, D, device=dev, dtype=torch.bfloat16) * 0.1
            o = torch.empty_like(q)
            sp = ops.wide_decode_splits(B, gnq, gkv, D, 1, ctx, win, 0)
            ws = torch.empty(ops.wide_decode_workspace_numel(B, gnq, gkv, D, 1, sp), device=dev)
            keys = min(ctx, win) if win else ctx
            ms = timeit(lambda i=0: ops.wide_decode_attention(q, kvl, gkv, bt, sl, o, window=win, softcap=50.0,
                                                              splits=sp, workspace=ws))
            report(f"wide_decode_attention_d{D}", ms, None, B * keys * gkv * D * 2 * 2,
                   {"B": B, "ctx": ctx, "window": win, "splits": sp})
            qp = torch.randn(2 * 2048, gnq, D, device=dev, dtype=torch.bfloat16) * 0.1
            op = torch.empty_like(qp)
            cu = [0, 2048, 4096]
            ts, tst = [t.to(dev) for t in ops.prefill_tiles(cu, [2048, 2048])]
            cuq = torch.tensor(cu, dtype=torch.int32, device=dev)
            cl = torch.tensor([2048, 2048], dtype=torch.int32, device=dev)
            ms = timeit(lambda i=0: ops.wide_prefill_attention(qp, kvl, gkv, bt[:2], cl, cuq, ts, tst, op,
                                                               window=win, softcap=50.0))
            # causal (or windowed) score + PV FLOPs of the two sequences
            pairs = sum(min(t + 1, win) if win else t + 1 for t in range(2048)) * 2
            report(f"wide_prefill_attention_d{D}", ms, 4.0 * pairs * gnq * D, None,
                   {"tokens": 4096, "window": win})
            del kvl

    if args.only and "wan" in args.only:
        # Wan2.1-T2V-1.3B: one guided DiT evaluation (batch 2) over a 17-frame 480 x 832 video latent
        # (5 x 60 x 104 -> 7,800 tokens per sample) and the VAE decode of 2 latent frames to 480 x 832
        from bloom_b200.models.wan import WanDiT, sampling_sigmas, wan_preset
        from bloom_b200.models.wan_vae import WanVAE, vae_preset

        wc = wan_preset("wan2.1-t2v-1.3b")
        dit = WanDiT(wc, dev)
        dit.random_init(0)
        ctx = (torch.randn(2, wc.text_len, wc.text_dim, device=dev) * 0.3).to(torch.bfloat16)
        text = dit.encode_text(ctx)
        lat = torch.randn(wc.in_dim, 5, 60, 104, device=dev)
        lb = lat.unsqueeze(0).expand(2, *lat.shape).contiguous()
        def eager_ms(fn, iters, warmup):  # host-built timestep inputs: not graph-capturable, time eagerly
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / iters

        ms = eager_ms(lambda: dit.velocity_tokens(lb, 500.0, text), 3, 2)
        S = 5 * 30 * 52
        T = 2 * S
        D, Fd, L = wc.dim, wc.ffn_dim, wc.text_len
        gemm_flops = 2.0 * T * wc.num_layers * (3 * D * D + D * D + D * D + D * D + 2 * D * Fd)
        attn_flops = 4.0 * 2 * wc.num_layers * (S * S + S * L) * D
        report("wan_dit_step_1.3b_cfg", ms, gemm_flops + attn_flops, None, {"tokens": T, "text_len": L})
        del dit, text
        vae = WanVAE(vae_preset("wan2.1"), dev)
        vae.random_init(0)
        z = torch.randn(16, 2, 60, 104, device=dev)
        ms = eager_ms(lambda: vae.decode(z), 2, 1)
        report("wan_vae_decode_2f_480x832", ms, None, None, {"frames": 2})
        del vae

    if args.only and "longcat" in args.only:
        # LongCat image-edit transformer, full width (3072, 24 heads): 2 joint + 4 single blocks
        # timed together and per block, 1,024 image tokens (512 x 512 image) + 512 text tokens
        import dataclasses as _dc

        from bloom_b200.models.longcat import LongCatTransformer, longcat_preset

        lc = _dc.replace(longcat_preset("longcat-image-edit"), num_layers=2, num_single_layers=4)
        tr = LongCatTransformer(lc, dev)
        tr.random_init(0)
        packed = torch.randn(1024, lc.in_channels, device=dev).to(torch.bfloat16)
        ctx = torch.randn(512, lc.joint_attention_dim, device=dev).to(torch.bfloat16)
        for _ in range(2):
            tr.forward(packed, ctx, 0.5, (32, 32))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            tr.forward(packed, ctx, 0.5, (32, 32))
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 3
        T, D = 1536, lc.dim
        blk = 2 * T * (3 * D * D + D * D + 2 * 4 * D * D) + 4 * T * T * D  # per block, both streams
        flops = 2 * blk + 4 * (2 * T * (3 * D * D + 4 * D * D + 5 * D * D) + 4 * T * T * D)
        report("longcat_transformer_2j4s_1536tok", ms, flops, None, {"tokens": T})
        del tr

    if not args.only or "norm" in args.only:
        for M in (256, 8192):
            x = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
            r = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
            w = torch.ones(H, device=dev, dtype=torch.bfloat16)
            out = torch.empty_like(x)
            ms = timeit(lambda i=0: ops.add_rmsnorm(x, r, w, 1e-5, out))
            report("add_rmsnorm", ms, None, M * H * 2 * 4, {"M": M})
            qkv = torch.randn(M, (nq + 2 * nkv) * hd, device=dev, dtype=torch.bfloat16)
            pos = torch.arange(M, device=dev, dtype=torch.int64)
            slots = torch.arange(M, device=dev, dtype=torch.int32)
            cache = torch.empty(1, M // 16 + 1, 2, nkv, 16, hd, device=dev, dtype=torch.bfloat16)
            cs = ops.rope_cos_sin(8192, hd, 5e5, dev)
            qo = torch.empty(M, nq, hd, device=dev, dtype=torch.bfloat16)
            ms = timeit(lambda i=0: ops.rope_kv_write(qkv, pos, slots, cs, qo, cache, 0, nq, nkv))
            report("rope_kv_write", ms, None, qkv.numel() * 4, {"M": M})
        logits = torch.randn(256, V // t, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda i=0: ops.argmax(logits))
        report("argmax", ms, None, logits.numel() * 2, {"B": 256})

    if not args.only or "sample" in args.only:
        # stochastic verify sampling: 64 sequences x (4 proposals + bonus) rows, temperature 0.8, top-p 0.9
        R = 320
        logits = torch.randn(R, V // t, device=dev, dtype=torch.bfloat16) * 3
        temp = torch.full((R,), 0.8, device=dev)
        topp = torch.full((R,), 0.9, device=dev)
        topk = torch.zeros(R, dtype=torch.int32, device=dev)
        seeds = torch.arange(R, dtype=torch.int64, device=dev)
        offs = torch.zeros(R, dtype=torch.int64, device=dev)
        draft = torch.randint(0, V // t, (R,), dtype=torch.int32, device=dev)
        ms = timeit(lambda i=0: ops.sample(logits, temp, topp, topk, seeds, offs, draft))
        report("verify_sample", ms, None, logits.numel() * 2, {"rows": R})

    if not args.only or "moe" in args.only:
        # Qwen3-30B-A3B expert FFN at EP=8: 16 local experts, 128 tokens x top-8, H 2048, I 768
        from bloom_b200.models.config import preset
        from bloom_b200.models.llama import DecoderLM, TPInfo
        from bloom_b200.models.qwen3_moe import MoEBlock

        cfg = preset("qwen3-moe-30b-a3b")
        cfg.num_layers = 1

        class _Shell:  # the MoE block only needs cfg / tp / device from its model
            pass

        sh = _Shell()
        sh.cfg, sh.device = cfg, dev
        sh.tp = TPInfo(rank=0, size=8)
        E, Hm, Im = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
        full = {"model.layers.0.mlp.gate.weight": torch.randn(E, Hm, device=dev, dtype=torch.bfloat16) * 0.02,
                "model.layers.0.mlp.experts.gate_proj": torch.randn(E, Im, Hm, device=dev, dtype=torch.bfloat16) * 0.02,
                "model.layers.0.mlp.experts.up_proj": torch.randn(E, Im, Hm, device=dev, dtype=torch.bfloat16) * 0.02,
                "model.layers.0.mlp.experts.down_proj": torch.randn(E, Hm, Im, device=dev, dtype=torch.bfloat16) * 0.02}
        blk = MoEBlock(sh, full)
        del full
        # routing alone: route (warp per token, register top-k) + plan
        from bloom_b200._ext import cuda as _cuda

        Cx = _cuda()
        K8, El8 = cfg.num_experts_per_tok, E // 8
        for Tm in (128, 512):
            lg = torch.randn(Tm, E, device=dev)
            ids = torch.empty(Tm, K8, dtype=torch.int32, device=dev)
            wts = torch.empty(Tm, K8, device=dev)
            slot = torch.empty(Tm, K8, dtype=torch.int32, device=dev)
            offs = torch.empty(El8 + 1, dtype=torch.int32, device=dev)
            mt = ((Tm * K8 + 15) // 16 + El8) * 12
            tg = torch.empty(mt, 4, dtype=torch.int32, device=dev)
            td = torch.empty_like(tg)
            ng = torch.zeros(1, dtype=torch.int32, device=dev)
            nd = torch.zeros_like(ng)
            cnt = torch.zeros(El8, dtype=torch.int32, device=dev)

            def route_plan(i=0):
                Cx.moe_route(lg, K8, True, 0, El8, ids, wts, slot, cnt)
                Cx.moe_plan(cnt, offs, 16, 12, 16, tg, ng, td, nd)

            report("moe_route_plan", timeit(route_plan), None, None, {"tokens": Tm})
        for Tm in (128, 4096):
            x = torch.randn(Tm, Hm, device=dev, dtype=torch.bfloat16)
            out = torch.empty_like(x)
            ms = timeit(lambda i=0: blk.forward(0, x, out))
            El = E // 8
            wbytes = El * 3 * Im * Hm * 2
            flops = 2.0 * Tm * cfg.num_experts_per_tok / 8 * 3 * Im * Hm
            report("moe_layer_ep8", ms, flops, wbytes, {"tokens": Tm, "local_experts": El})

    if not args.only or "quant" in args.only:
        # GGUF decode GEMV straight from the block-quantised rows (Llama-3-8B gate_up / down
        # rows at M = 1 and 8 tokens); bytes = the quantised weight planes
        for kind in ("Q8_0", "Q4_0"):
            for nm, N, K in (("gate_up", 2 * I // t, H), ("down", H, I // t)):
                nrot = max(1, int(math.ceil(400e6 / (N * K))))
                qw = [ops.QWeight(kind, (torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8) if kind == "Q8_0"
                                         else torch.randint(0, 256, (N, K // 2), device=dev, dtype=torch.uint8)),
                                  torch.full((N, K // 32), 0.01, device=dev, dtype=torch.float16), K)
                      for _ in range(nrot)]
                for M in (1, 8):
                    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
                    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                    ms = timeit(lambda i=0: ops.gemm(x, qw[i % nrot], out))
                    report(f"qgemv_{kind}_{nm}", ms, 2.0 * M * N * K, qw[0].nbytes() + M * K * 2, {"M": M, "N": N, "K": K})
                del qw

    if args.json:
        with open(args.json, "w") as f:
            json.dump({"peaks": {"hbm_gbs": hbm, "bf16_tflops": tfl, "source": src}, "rows": rows}, f, indent=1)


if __name__ == "__main__":
    main()
