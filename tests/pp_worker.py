"""Worker for the pipeline-parallel GPU test (launched by tests/test_pp_gpu.py
through torchrun): every rank is one pipeline stage of the same 4-layer
model; greedy generation through the engine must track the fp32 oracle and
every stage must see the same tokens."""
import dataclasses
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bloom_b200 import ops  # noqa: E402
from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from bloom_b200.models.config import preset  # noqa: E402
from bloom_b200.models.llama import DecoderLM  # noqa: E402
from bloom_b200.models.reference import forward_logits, random_weights  # noqa: E402
from bloom_b200.parallel.comm import init_distributed  # noqa: E402
from bloom_b200.parallel.pipeline import pipeline_from_world  # noqa: E402


def main():
    rank, world, local = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    cfg = dataclasses.replace(preset("tiny-llama"), num_layers=4)
    w = random_weights(cfg, seed=5, std=0.08, device=dev)
    pp = pipeline_from_world()
    model = DecoderLM(cfg, None, dev, pp=pp)
    model.shard_full(w)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=64, max_model_len=512,
                                        num_blocks=128, use_cuda_graphs=True, autotune=False))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 33, 90, 1)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True))
    worst = 0.0
    for p, o in zip(prompts, outs):
        logits = forward_logits(cfg, w, list(p) + o.token_ids)
        for j, tok in enumerate(o.token_ids):
            row = logits[len(p) - 1 + j]
            spread = (row.max() - row.median()).item()
            worst = max(worst, (row.max() - row[tok]).item() / max(spread, 1e-6))
    souts = eng.generate(prompts, SamplingParams(max_tokens=6, temperature=0.8, top_p=0.9, seed=11, ignore_eos=True))
    toks = torch.tensor([t for o in outs + souts for t in o.token_ids], device=dev)
    allt = [torch.empty_like(toks) for _ in range(world)]
    dist.all_gather(allt, toks)
    res = {"rank": rank, "layers": [model.l0, model.l1], "kv_layers": int(eng.runner.kv_cache.shape[0]),
           "worst_gap": worst, "ok": worst < 0.03, "ranks_agree": all(torch.equal(allt[0], t) for t in allt),
           "status": int(ops.status(local)[0].item()), "graphs": eng.runner.use_cuda_graphs}
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
