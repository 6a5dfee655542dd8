"""bloom_server: python -m bloom_b200.server --model PATH|PRESET [--host 127.0.0.1 --port 3000]

Flags follow the reference server CLI (crates/server/src/cli.rs:18-327):
--host/--port (127.0.0.1:3000), --max-concurrent 4, --context-size 2048,
--api-key (repeatable; also BLOOM_API_KEYS comma-separated), --cors-origin,
--device, --speculative/--draft-model/--num-speculative-tokens, --doctor
(side-effect-free environment report).  --tp N runs tensor parallel when the
server is launched with torchrun (rank 0 serves HTTP; other ranks follow).
"""
from __future__ import annotations

import argparse
import json
import os
import sys


def build_parser():
    ap = argparse.ArgumentParser(prog="bloom_server")
    ap.add_argument("--model", "-m")
    ap.add_argument("--host", default=os.environ.get("BLOOM_HOST", "127.0.0.1"))
    ap.add_argument("--port", type=int, default=int(os.environ.get("BLOOM_PORT", "3000")))
    ap.add_argument("--max-concurrent", type=int, default=4)
    ap.add_argument("--context-size", type=int, default=2048)
    ap.add_argument("--api-key", action="append", default=[])
    ap.add_argument("--cors-origin", action="append", default=[])
    ap.add_argument("--device", choices=["cpu", "gpu"], default="gpu")
    ap.add_argument("--speculative", choices=["none", "ngram", "draft"], default="none")
    ap.add_argument("--draft-model")
    ap.add_argument("--num-speculative-tokens", type=int, default=5)
    ap.add_argument("--model-id")
    ap.add_argument("--max-resident-models", type=int, default=int(os.environ.get("BLOOM_MAX_RESIDENT_MODELS", "1")),
                    help="models kept loaded at once (requests select one with their `model` field)")
    ap.add_argument("--memory-host-limit", type=int, default=0,
                    help="host bytes all resident models may hold (0 = physical RAM)")
    ap.add_argument("--memory-device-limit", type=int, default=0,
                    help="device bytes all resident models may hold (0 = every GPU's memory)")
    ap.add_argument("--doctor", action="store_true")
    ap.add_argument("--doctor-format", choices=["text", "json"], default="text")
    ap.add_argument("--models-dir", default=os.environ.get("BLOOM_MODELS_DIR"),
                    help="catalog for /v1/model-management (list, preflight, switch, unload, remove)")
    ap.add_argument("--pipeline", action="store_true",
                    help="under torchrun: the ranks are pipeline stages (layer ranges) instead of tensor-parallel shards")
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused",
                    help="tensor-parallel collectives (torchrun launches): fused NVLink kernels or NCCL")
    ap.add_argument("--enable-ifb", action="store_true", default=True,
                    help="in-flight batching (always on for the GPU engine)")
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if args.doctor:
        from ..utils.doctor import doctor_report

        keys = list(args.api_key) + [k for k in os.environ.get("BLOOM_API_KEYS", "").split(",") if k]
        rep = doctor_report(args.model, speculative=args.speculative, draft_model=args.draft_model,
                            context_size=args.context_size, max_concurrent=args.max_concurrent, host=args.host,
                            api_keys=keys)
        if args.doctor_format == "json":
            print(json.dumps(rep, indent=2))
        else:
            from ..utils.doctor import render_text

            print(render_text(rep), end="")
        return 1 if rep["status"] == "fail" else 0
    if not args.model:
        print("error: --model is required", file=sys.stderr)
        return 2
    keys = list(args.api_key) + [k for k in os.environ.get("BLOOM_API_KEYS", "").split(",") if k]
    if args.host not in ("127.0.0.1", "localhost", "::1") and not keys:
        print("error: refusing to listen on a non-loopback address without --api-key", file=sys.stderr)
        return 2
    from ..engine.pipeline import InferencePipeline
    from .app import ServerSettings, create_app
    from .runtime import ServingRuntime, TPControl, follower_loop

    tp_info, pp_info, ctrl = None, None, None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:  # launched by torchrun: tensor parallel over the ranks
        from ..models.llama import TPInfo
        from ..models.config import PRESETS, preset
        from ..parallel.comm import Communicator, init_distributed
        import torch
        import torch.distributed as dist

        rank, world, local = init_distributed("nccl")
        dev = torch.device("cuda", local)
        if args.pipeline:
            from ..parallel.pipeline import pipeline_from_world

            pp_info = pipeline_from_world()
        else:
            hidden = preset(args.model).hidden_size if args.model in PRESETS else 8192
            comm = Communicator(rank, world, dev, dist.group.WORLD, mode=args.comm,
                                max_tokens=max(args.context_size, 8192), hidden=hidden)
            tp_info = TPInfo(rank=rank, size=world, group=dist.group.WORLD, comm=comm)
        ctrl = TPControl()
    pipe = InferencePipeline.load(args.model, device=args.device, context_size=args.context_size,
                                  speculative=args.speculative, draft_model=args.draft_model,
                                  num_speculative_tokens=args.num_speculative_tokens,
                                  max_num_seqs=max(4, args.max_concurrent), tp_info=tp_info, pp_info=pp_info)
    if ctrl is not None and ctrl.rank != 0:
        follower_loop(pipe.llm, ctrl)  # returns when rank 0 shuts down
        return 0
    mid = args.model_id or os.path.basename(str(args.model).rstrip("/"))
    settings = ServerSettings(model_id=mid, api_keys=keys, context_size=pipe.context_size,
                              max_concurrent=args.max_concurrent, cors_origins=args.cors_origin,
                              models_dir=args.models_dir, pool_capacity=args.max_resident_models,
                              memory_host_limit=args.memory_host_limit, memory_device_limit=args.memory_device_limit)
    runtime = ServingRuntime(pipe, mid, args.max_concurrent, ctrl=ctrl) if ctrl is not None else None
    app = create_app(pipe, settings, runtime)
    if ctrl is None:  # model switching re-loads on this process's device (not offered under tensor parallel)
        app.state.model_loader = lambda path: InferencePipeline.load(
            path, device=args.device, context_size=args.context_size, max_num_seqs=max(4, args.max_concurrent))
    import uvicorn

    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="warning")
    finally:
        if runtime is not None:
            runtime.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
