"""Worker for the tensor-parallel GPU test (launched by tests/test_tp_gpu.py through torchrun).

Every rank builds the same tiny model sharded over the group, runs greedy
generation through the engine and checks it against the fp32 oracle."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bloom_b200 import ops  # noqa: E402
from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from bloom_b200.models.config import preset  # noqa: E402
from bloom_b200.models.llama import DecoderLM, TPInfo  # noqa: E402
from bloom_b200.models.reference import forward_logits, random_weights  # noqa: E402
from bloom_b200.parallel.comm import Communicator, init_distributed  # noqa: E402


def main():
    mode = sys.argv[1] if len(sys.argv) > 1 else "nccl"
    graphs = (sys.argv[2] == "graphs") if len(sys.argv) > 2 else True
    name = sys.argv[3] if len(sys.argv) > 3 else "tiny-tp"
    rank, world, local = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    cfg = preset(name)
    w = random_weights(cfg, seed=3, std=0.08, device=dev)
    comm = Communicator(rank, world, dev, dist.group.WORLD, mode, max_tokens=512, hidden=cfg.hidden_size,
                        timeout_s=10.0)
    model = DecoderLM(cfg, TPInfo(rank, world, dist.group.WORLD, comm), dev)
    model.shard_full(w)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=512,
                                        num_blocks=128, use_cuda_graphs=graphs))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 33, 70, 1)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True))
    ok = True
    worst = 0.0
    for p, o in zip(prompts, outs):
        logits = forward_logits(cfg, w, list(p) + o.token_ids)
        for j, tok in enumerate(o.token_ids):
            row = logits[len(p) - 1 + j]
            spread = (row.max() - row.median()).item()
            gap = (row.max() - row[tok]).item()
            worst = max(worst, gap / max(spread, 1e-6))
            if gap > 0.03 * spread + 1e-4:
                ok = False
    # stochastic rows: the full-vocabulary rows are gathered from the shards
    # (fused: one P2P kernel) and sampled with the same Philox stream on every rank
    souts = eng.generate(prompts, SamplingParams(max_tokens=6, temperature=0.8, top_p=0.9, seed=11, ignore_eos=True))
    toks = torch.tensor([t for o in outs + souts for t in o.token_ids], device=dev)
    allt = [torch.empty_like(toks) for _ in range(world)]
    dist.all_gather(allt, toks)
    same = all(torch.equal(allt[0], t) for t in allt)
    status = int(ops.status(local)[0].item())
    # guard words around every symmetric buffer: a stray P2P store by any rank shows up here
    canaries = comm.fused.check_canaries() if comm.fused is not None else {}
    bad = torch.tensor([sum(canaries.values())], device=dev)
    dist.all_reduce(bad)
    eng.shutdown()
    if rank == 0:
        print(json.dumps({"ok": ok, "ranks_agree": same, "worst_gap": worst, "status": status,
                          "graph_steps": eng.runner.stats["graph_steps"], "bad_guard_words": int(bad.item()),
                          "guards_checked": sorted(canaries)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if (ok and same and status == 0 and int(bad.item()) == 0) else 1)


if __name__ == "__main__":
    main()
