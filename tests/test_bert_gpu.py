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


def test_minilm_fp32_matches_reference_closely():
    """The fp32 path (fp32 kernels + fp32 SGEMM) agrees with the fp32 oracle to
    fp32 rounding, far tighter than the bf16 path."""
    from bloom_b200.models.bert import BertEmbedder, reference_embed
    from bloom_b200.models.config import preset

    cfg = preset("minilm-l6")
    sd = BertEmbedder.random_state_dict(cfg, seed=2, std=0.05)
    e = BertEmbedder(cfg, "cuda", dtype=torch.float32)
    e.load_state_dict(sd)
    rng = random.Random(3)
    seqs = [[rng.randrange(cfg.vocab_size) for _ in range(rng.randint(16, 128))] for _ in range(21)] + [[101, 102]]
    got = e.forward_ids(seqs)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    exp = reference_embed(cfg, sd, seqs, device="cuda")
    torch.backends.cuda.matmul.allow_tf32 = prev
    assert (got - exp).abs().max().item() < 1e-4


def test_gemm_gelu_epilogue():
    from bloom_b200 import ops

    x = torch.randn(77, 384, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(1536, 384, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(1536, device="cuda", dtype=torch.bfloat16)
    y = ops.gemm(x, w, epi=ops.EPI_GELU, bias=b)
    ref = torch.nn.functional.gelu(x.float() @ w.float().t() + b.float())
    assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2


@pytest.mark.parametrize("hd", [32, 64])
def test_varlen_attention_tensor_core_matches_fp32(hd):
    """Non-causal varlen attention (mma.sync tiles) against an fp32 softmax,
    over odd lengths including 1, a partial 16-key tile and 512."""
    import torch

    from bloom_b200 import ops

    torch.manual_seed(hd)
    lens = [1, 17, 100, 64, 129, 512]
    NH = 12 if hd == 32 else 6
    cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), dtype=torch.int32, device="cuda")
    T = int(cu[-1])
    qkv = torch.randn(T, 3 * NH * hd, device="cuda").to(torch.bfloat16)
    scale = hd ** -0.5
    out = ops.varlen_attention(qkv, cu, NH, hd, max(lens), scale)
    q, k, v = qkv.float().view(T, 3, NH, hd).unbind(1)
    worst = 0.0
    for i, L in enumerate(lens):
        a, b = int(cu[i]), int(cu[i + 1])
        s = torch.einsum("qhd,khd->hqk", q[a:b], k[a:b]) * scale
        ref = torch.einsum("hqk,khd->qhd", s.softmax(-1), v[a:b]).reshape(L, NH * hd)
        worst = max(worst, (out[a:b].float() - ref).abs().max().item())
    assert worst < 2e-2, worst
