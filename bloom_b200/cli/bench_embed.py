"""Embedding throughput benchmark: MiniLM-L6 shape, 1 GPU or data parallel.

    python -m bloom_b200.cli.bench_embed [--steps K] [--warmup W]
    torchrun --nproc-per-node 8 -m bloom_b200.cli.bench_embed          (DP = 8)
    ... --dtype fp32      full precision (fp32 weights, activations and arithmetic)

Workload per step: 256 sequences per GPU with lengths uniform in [16, 128],
uniform-random token ids, mean pooling and L2 normalisation (random N(0,0.02)
weights, seed 0).  Data parallel: every rank holds a full model replica and
embeds its own 256 sequences; the step time is the max over ranks (device
time, CUDA events) and the value is total embeddings/s for all GPUs.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import sys


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--dtype", choices=("bf16", "fp32"), default="bf16",
                    help="fp32: full-precision weights and activations (the model config's stated precision)")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist

    from bloom_b200.models.bert import BertEmbedder
    from bloom_b200.models.config import preset
    from bloom_b200.parallel.comm import init_distributed

    rank, world, local = init_distributed("nccl")
    dev = torch.device("cuda", local)
    cfg = preset("minilm-l6")
    e = BertEmbedder(cfg, dev, dtype=torch.float32 if args.dtype == "fp32" else torch.bfloat16)
    e.load_state_dict(BertEmbedder.random_state_dict(cfg, seed=0))
    rng = random.Random(1000 + rank)

    def batch():
        lens = [rng.randint(16, 128) for _ in range(args.batch)]
        ids = [rng.randrange(cfg.vocab_size) for L in lens for _ in range(L)]
        pos = [p for L in lens for p in range(L)]
        cu = [0]
        for L in lens:
            cu.append(cu[-1] + L)
        return (torch.tensor(ids, dtype=torch.int32).pin_memory(), torch.tensor(pos, dtype=torch.int32).pin_memory(),
                torch.tensor(cu, dtype=torch.int32).pin_memory(), max(lens))

    batches = [batch() for _ in range(args.steps + args.warmup)]

    def run(b):
        ids, pos, cu, ml = b
        out = e.forward_packed(ids.to(dev, non_blocking=True), pos.to(dev, non_blocking=True),
                               cu.to(dev, non_blocking=True), ml)
        return out.to("cpu", non_blocking=True)

    for b in batches[:args.warmup]:
        run(b)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ts = []
    for b in batches[args.warmup:]:
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run(b)
        z.record()
        z.synchronize()
        ts.append(a.elapsed_time(z))
    t = torch.tensor([sum(ts)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = t.item()
    value = args.batch * world * args.steps / (total_ms / 1e3)
    if rank == 0:
        print(json.dumps({"metric": "embeddings/s (MiniLM-L6 shape, 256 seqs/GPU, len U[16,128])",
                          "value": round(value, 1), "unit": "embeddings/s (all GPUs)", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3),
                          "parallelism": f"dp{world}", "dtype": args.dtype, "data": "synthetic",
                          "includes": "H2D of ids from pinned memory, D2H of embeddings"}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
