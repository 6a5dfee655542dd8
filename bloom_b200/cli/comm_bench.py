"""Tensor-parallel collective benchmark: the fused NVLink kernels against NCCL.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m bloom_b200.cli.comm_bench [--tokens 8,64,256,1024,8192] [--hidden 4096]

For every token count T it times, on every rank, and prints the maximum over
ranks (one JSON line per case, rank 0):

  coll_push    tp_allreduce_rmsnorm on partials the GEMM already pushed
               (local slot sum + residual + RMSNorm + all-gather over NVLink)
  coll_pull    the same kernel reading the peers' partials (P2P loads)
  nccl_coll    NCCL all-reduce of the [T, H] partial + the add_rmsnorm kernel
  <gemm>_fused a row-parallel GEMM (o_proj [H, H/N] or down [H, F/N] of the
               Llama-3-8B shape) whose epilogue pushes rows to their owners,
               then coll_push
  <gemm>_nccl  the same GEMM into a local buffer, NCCL all-reduce, add_rmsnorm
  mlp_chain    the tensor-parallel part of a decoder layer's second half:
               o_proj (push) -> collective -> gate_up + SwiGLU -> down (push)
               -> collective -> next qkv GEMM, with the all-gather waited
               for in the collective (mlp_chain) or deferred to the GEMM that
               reads the rows (mlp_chain_deferred), and on NCCL (mlp_chain_nccl)

Each case is captured as a CUDA graph of `--iters` back-to-back ops and
replayed (warm-up replays first); the time is CUDA events on the launching
stream / iters, median of the timed replays.  Inputs are hot in L2 (a decode
step's partials are too).  `nvlink_bytes` is what one rank must send over
NVLink per op; `floor_us` is the larger of that at the measured 770 GB/s
peer-copy bandwidth and the GEMM FLOPs at the measured bf16 peak.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops", 1590.0)), float(d.get("hbm_gbs", 6650.0))
    except (OSError, ValueError):
        return 1590.0, 6650.0


def _time_graph(fn, iters: int, reps: int = 7, warm: int = 3) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # eager warm-up (lazy allocations, autotune)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    for _ in range(warm):
        g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1000.0 / iters)
    del g
    return statistics.median(times)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="8,64,256,1024,8192")
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--iters", type=int, default=32)
    ap.add_argument("--out", default="")
    ap.add_argument("--trace", action="store_true",
                    help="also print the phase timeline of block 0 (entry, ready, rows written, done)")
    args = ap.parse_args(argv)

    from bloom_b200 import ops
    from bloom_b200.parallel.comm import init_distributed
    from bloom_b200.parallel.fused import FusedComm

    rank, world, local = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    H, F = args.hidden, args.ffn
    tokens = [int(t) for t in args.tokens.split(",")]
    Tmax = max(tokens)
    fc = FusedComm(rank, world, dev, dist.group.WORLD, max_tokens=Tmax, hidden=H, timeout_s=5.0)
    tflops, hbm = _peaks()
    g = torch.Generator(device=dev).manual_seed(rank)
    norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    resid = torch.randn(Tmax, H, device=dev, dtype=torch.bfloat16, generator=g)
    part = torch.randn(Tmax, H, device=dev, dtype=torch.bfloat16, generator=g) * 0.01
    fc.partial(Tmax).copy_(part)
    weights = {"o_proj": torch.randn(H, H // world, device=dev, dtype=torch.bfloat16, generator=g) * 0.02,
               "down": torch.randn(H, F // world, device=dev, dtype=torch.bfloat16, generator=g) * 0.02}
    w_gu = torch.randn(2 * F // world, H, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    w_qkv = torch.randn((H + 2 * H // 4) // world, H, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    acts = {k: torch.randn(Tmax, w.shape[1], device=dev, dtype=torch.bfloat16, generator=g) for k, w in weights.items()}
    results = []

    def report(case, T, us, gemm_flops=0.0, nv_bytes=0.0):
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        floor = max(nv_bytes / (PEER_GBS * 1e3), gemm_flops / (tflops * 1e6))
        r = {"case": case, "world": world, "T": T, "H": H, "us": round(float(t.item()), 2),
             "nvlink_bytes": int(nv_bytes), "floor_us": round(floor, 2),
             "frac_of_floor": round(floor / float(t.item()), 3) if floor > 0 else None}
        results.append(r)
        if rank == 0:
            print(json.dumps(r), flush=True)

    for T in tokens:
        rows = (T + world - 1) // world
        ag_bytes = rows * (world - 1) * H * 2  # this rank's normalised rows to every peer
        rs_bytes = (T - rows) * H * 2  # the GEMM pushes the other ranks' rows (reduce-scatter)
        r_T = resid[:T]
        report("coll_push", T, _time_graph(lambda: fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=True),
                                           args.iters), 0.0, ag_bytes)
        report("coll_pull", T, _time_graph(lambda: fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=False),
                                           args.iters), 0.0, ag_bytes + rs_bytes)
        if args.trace:
            from bloom_b200._ext import cuda

            cap = 64
            tb = torch.zeros(cap * 4, dtype=torch.int64, device=dev)
            cuda().tp_ar_set_trace(tb)
            fn = (lambda: fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=True))
            _time_graph(fn, cap)
            cuda().tp_ar_set_trace(None)
            tr = tb.view(cap, 4).cpu().double()
            ok = (tr > 0).all(1)
            tr = tr[ok]
            if tr.shape[0] > 2:
                order = tr[:, 0].argsort()
                tr = tr[order]
                ph = {"ready_us": (tr[:, 1] - tr[:, 0]), "rows_us": (tr[:, 2] - tr[:, 1]),
                      "done_us": (tr[:, 3] - tr[:, 2]), "period_us": (tr[1:, 0] - tr[:-1, 0])}
                med = {k: round(float(v.median()) / 1000.0, 2) for k, v in ph.items()}
                allm = [None] * world
                dist.all_gather_object(allm, med)
                if rank == 0:
                    print(json.dumps({"case": "coll_push_trace", "world": world, "T": T, "per_rank": allm}),
                          flush=True)
        buf = part[:T].clone()
        xo = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

        def nccl_coll():
            dist.all_reduce(buf)
            ops.add_rmsnorm(buf, r_T, norm_w, 1e-5, out=xo)

        report("nccl_coll", T, _time_graph(nccl_coll, args.iters), 0.0, ag_bytes + rs_bytes)
        for name, w in weights.items():
            x = acts[name][:T]
            flops = 2.0 * T * w.shape[0] * w.shape[1]
            out_local = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

            def fused_op():
                ops.gemm(x, w, fc.partial(T), push=fc.push_args(T))
                fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=True)

            def nccl_op():
                ops.gemm(x, w, out_local)
                dist.all_reduce(out_local)
                ops.add_rmsnorm(out_local, r_T, norm_w, 1e-5, out=xo)

            report(f"{name}_fused", T, _time_graph(fused_op, args.iters), flops, ag_bytes + rs_bytes)
            report(f"{name}_nccl", T, _time_graph(nccl_op, args.iters), flops, ag_bytes + rs_bytes)
        # decoder-layer chain with and without the deferred all-gather
        x_o = acts["o_proj"][:T]
        chain_flops = 2.0 * T * H * (H // world + 2 * F // world + F // world + w_qkv.shape[0])

        def chain(defer):
            ops.gemm(x_o, weights["o_proj"], fc.partial(T), push=fc.push_args(T))
            x = fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=True, defer=defer)
            act = ops.gemm(x, w_gu, epi=ops.EPI_SWIGLU, wait=fc.wait_args() if defer else None)
            ops.gemm(act, weights["down"], fc.partial(T), push=fc.push_args(T))
            x = fc.allreduce_rmsnorm(T, r_T, norm_w, 1e-5, pushed=True, defer=defer)
            ops.gemm(x, w_qkv, wait=fc.wait_args() if defer else None)

        def chain_nccl():
            y = ops.gemm(x_o, weights["o_proj"])
            dist.all_reduce(y)
            x = ops.add_rmsnorm(y, r_T, norm_w, 1e-5)
            act = ops.gemm(x, w_gu, epi=ops.EPI_SWIGLU)
            y = ops.gemm(act, weights["down"])
            dist.all_reduce(y)
            x = ops.add_rmsnorm(y, r_T, norm_w, 1e-5)
            ops.gemm(x, w_qkv)

        report("mlp_chain", T, _time_graph(lambda: chain(False), args.iters), chain_flops, 2 * (ag_bytes + rs_bytes))
        report("mlp_chain_deferred", T, _time_graph(lambda: chain(True), args.iters), chain_flops,
               2 * (ag_bytes + rs_bytes))
        report("mlp_chain_nccl", T, _time_graph(chain_nccl, args.iters), chain_flops, 2 * (ag_bytes + rs_bytes))
    st = int(ops.status(local)[0].item())
    bad = sum(fc.check_canaries().values())
    if rank == 0:
        print(json.dumps({"status": st, "bad_guard_words": bad}), flush=True)
        if args.out:
            with open(args.out, "w") as f:
                json.dump(results, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
