"""BERT/MiniLM embeddings on the GPU vs the fp32 PyTorch oracle."""
import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_minilm_embeddings_match_reference():
    from bloom_b200.models.bert import BertEmbedder, reference_embed
    from bloom_b200.models.config import preset

    cfg = preset("minilm-l6")
    sd = BertEmbedder.random_state_dict(cfg, seed=1, std=0.05)
    e = BertEmbedder(cfg, "cuda")
    e.load_state_dict(sd)
    rng = random.Random(0)
    seqs = [[rng.randrange(cfg.vocab_size) for _ in range(rng.randint(16, 128))] for _ in range(37)]
    seqs.append([101, 102])
    got = e.forward_ids(seqs)
    exp = reference_embed(cfg, sd, seqs, device="cuda")
    assert got.shape == (len(seqs), cfg.hidden_size)
    norms = got.norm(dim=1)
    assert torch.allclose(norms, torch.ones_like(norms), atol=1e-3)
    cos = (got * exp).sum(1)
    assert cos.min().item() > 0.995, cos.min().item()


def test_gemm_gelu_epilogue():
    from bloom_b200 import ops

    x = torch.randn(77, 384, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(1536, 384, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(1536, device="cuda", dtype=torch.bfloat16)
    y = ops.gemm(x, w, epi=ops.EPI_GELU, bias=b)
    ref = torch.nn.functional.gelu(x.float() @ w.float().t() + b.float())
    assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2
