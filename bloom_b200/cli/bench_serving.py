"""Serving benchmark through the OpenAI-compatible HTTP server, tensor parallel.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bloom_b200.cli.bench_serving \\
        --model llama3-70b --draft-model llama3-1b-draft --spec-len 4 \\
        --requests 64 --prompt-len 4096 --output-len 512 --stream 8

Every rank builds its shard of the model (random init of the named shape);
rank 0 also holds the draft model, serves HTTP on 127.0.0.1 and runs the
client: all requests go to /v1/completions with token-id prompts (uniform
random ids, greedy, min_tokens = max_tokens so every request produces the full
output), the first --stream of them with stream=true.  The other ranks follow
rank 0's engine steps.  Prints one JSON line: output tokens/s of the whole
run (wall clock on rank 0, which includes HTTP and streaming), p50 / p90 time
to first token of the streamed requests, and the speculation acceptance.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import os
import statistics
import sys
import threading
import time


async def _client(port, model_id, prompts, out_len, n_stream):
    import aiohttp

    url = f"http://127.0.0.1:{port}/v1/completions"
    res = []

    async def one(i, p, session):
        body = {"model": model_id, "prompt": p, "max_tokens": out_len, "min_tokens": out_len, "temperature": 0.0,
                "stream": i < n_stream}
        t0 = time.perf_counter()
        ttft = None
        ntok = 0
        async with session.post(url, json=body) as r:
            if r.status != 200:
                raise RuntimeError(f"HTTP {r.status}: {await r.text()}")
            if body["stream"]:
                async for raw in r.content:
                    line = raw.decode().strip()
                    if not line.startswith("data: ") or line == "data: [DONE]":
                        continue
                    if ttft is None:
                        ttft = time.perf_counter() - t0
                    ntok += 1
            else:
                d = await r.json()
                ntok = d["usage"]["completion_tokens"]
        res.append({"i": i, "stream": body["stream"], "ttft_s": ttft, "total_s": time.perf_counter() - t0,
                    "tokens": ntok})

    timeout = aiohttp.ClientTimeout(total=3600)
    async with aiohttp.ClientSession(timeout=timeout) as session:
        await asyncio.gather(*(one(i, p, session) for i, p in enumerate(prompts)))
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="bench_serving")
    ap.add_argument("--model", default="llama3-70b")
    ap.add_argument("--draft-model", default="llama3-1b-draft")
    ap.add_argument("--spec-len", type=int, default=4)
    ap.add_argument("--speculative", default="draft", choices=["none", "ngram", "draft"])
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=4096)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--stream", type=int, default=8)
    ap.add_argument("--port", type=int, default=3917)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--warmup-requests", type=int, default=4)
    a = ap.parse_args(argv)

    import torch
    import torch.distributed as dist

    from ..engine.pipeline import InferencePipeline
    from ..models.config import preset
    from ..models.llama import TPInfo
    from ..parallel.comm import Communicator, init_distributed
    from ..server.app import ServerSettings, create_app
    from ..server.runtime import ServingRuntime, TPControl, follower_loop

    rank, world, local = init_distributed("nccl" if torch.cuda.is_available() else "gloo")
    dev = torch.device("cuda", local)
    ctx = a.prompt_len + a.output_len + a.spec_len + 16
    tp_info, ctrl = None, None
    if world > 1:
        comm = Communicator(rank, world, dev, dist.group.WORLD, mode=a.comm, max_tokens=max(ctx, 8192),
                            hidden=preset(a.model).hidden_size)
        tp_info = TPInfo(rank=rank, size=world, group=dist.group.WORLD, comm=comm)
        ctrl = TPControl()
    t0 = time.perf_counter()
    pipe = InferencePipeline.load(a.model, device="gpu", context_size=ctx, speculative=a.speculative,
                                  draft_model=a.draft_model if a.speculative == "draft" else None,
                                  num_speculative_tokens=a.spec_len, max_num_seqs=a.requests, tp_info=tp_info)
    init_s = time.perf_counter() - t0
    if ctrl is not None and rank != 0:
        follower_loop(pipe.llm, ctrl)
        dist.barrier()
        return 0
    mid = a.model
    runtime = ServingRuntime(pipe, mid, a.requests + a.warmup_requests, ctrl=ctrl)
    app = create_app(pipe, ServerSettings(model_id=mid, context_size=ctx, max_concurrent=a.requests + 4), runtime)
    import uvicorn

    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=a.port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)
    g = torch.Generator().manual_seed(1234)
    V = pipe.cfg.vocab_size
    warm = [torch.randint(3, V, (256,), generator=g).tolist() for _ in range(a.warmup_requests)]
    asyncio.run(_client(a.port, mid, warm, 16, 1))
    prompts = [torch.randint(3, V, (a.prompt_len,), generator=g).tolist() for _ in range(a.requests)]
    spec0 = pipe.llm.speculator.stats(pipe.llm) if pipe.llm.speculator is not None else None
    t1 = time.perf_counter()
    res = asyncio.run(_client(a.port, mid, prompts, a.output_len, a.stream))
    wall = time.perf_counter() - t1
    spec = pipe.llm.speculator.stats(pipe.llm) if pipe.llm.speculator is not None else None
    server.should_exit = True
    th.join(timeout=30)
    runtime.shutdown()
    total_tokens = sum(r["tokens"] for r in res if not r["stream"]) + sum(
        a.output_len for r in res if r["stream"])  # streamed chunk counts can merge tokens; each got output_len
    ttfts = sorted(r["ttft_s"] * 1e3 for r in res if r["stream"] and r["ttft_s"] is not None)
    line = {
        "metric": "output tok/s over HTTP (64 concurrent, 8 streamed), Llama-3-70B-shape TP + 1B-draft speculation",
        "value": round(total_tokens / wall, 1), "unit": "output tokens/s (whole box, wall clock incl. HTTP)",
        "n_gpus": world, "wall_s": round(wall, 2), "requests": a.requests, "streamed": a.stream,
        "p50_ttft_ms_streamed": round(statistics.median(ttfts), 1) if ttfts else None,
        "p90_ttft_ms_streamed": round(ttfts[int(0.9 * (len(ttfts) - 1))], 1) if ttfts else None,
        "config": {"model": a.model, "draft": a.draft_model if a.speculative == "draft" else None,
                   "speculative": a.speculative, "spec_len": a.spec_len, "prompt_len": a.prompt_len,
                   "output_len": a.output_len, "parallelism": f"tp{world}", "comm": a.comm if world > 1 else "none",
                   "dtype": "bf16", "data": "synthetic token ids, random-init weights"},
        "init_s": round(init_s, 1),
    }
    if spec is not None and spec0 is not None:
        d_acc = spec["accepted"] - spec0["accepted"]
        d_prop = spec["proposed"] - spec0["proposed"]
        d_grp = spec["verify_groups"] - spec0["verify_groups"]
        line["speculation"] = {"acceptance_rate": round(d_acc / d_prop, 4) if d_prop else 0.0,
                               "tokens_per_verify": round((d_acc + d_grp) / d_grp, 3) if d_grp else 0.0}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
    return 0


if __name__ == "__main__":
    sys.exit(main())
