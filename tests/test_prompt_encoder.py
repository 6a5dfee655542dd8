"""LongCat text prompt encoder: the edit chat template (host) and the paged
decoder's final-normed hidden states against the fp32 oracle (GPU)."""
import pytest
import torch


def test_edit_prompt_template():
    from bloom_b200.models.prompt_encoder import EDIT_SYSTEM, edit_prompt_text

    t = edit_prompt_text("make the sky red")
    assert t.startswith("<|im_start|>system\n" + EDIT_SYSTEM + "<|im_end|>\n<|im_start|>user\n")
    assert t.endswith("make the sky red<|im_end|>\n<|im_start|>assistant\n")
    assert "<|vision_start|>" not in t
    v = edit_prompt_text("x", image_tokens=3)
    assert "<|vision_start|>" + "<|image_pad|>" * 3 + "<|vision_end|>x<|im_end|>" in v


def test_oracle_hidden_is_the_normed_stream():
    from bloom_b200.models.config import preset
    from bloom_b200.models.prompt_encoder import reference_hidden
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-qwen2")
    w = random_weights(cfg, seed=1)
    h = reference_hidden(cfg, w, [5, 9, 11, 2])
    assert h.shape == (4, cfg.hidden_size)
    # RMSNorm output times the norm weight: rms of h / w is one per row
    r = (h / w["model.norm.weight"].float()).pow(2).mean(-1).sqrt()
    assert torch.allclose(r, torch.ones_like(r), atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [7, 40, 300])
def test_prompt_encoder_matches_oracle(T):
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM
    from bloom_b200.models.prompt_encoder import TextPromptEncoder, reference_hidden
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-qwen2")
    w = random_weights(cfg, seed=3, device="cuda")
    m = DecoderLM(cfg, device=torch.device("cuda:0"))
    m.shard_full(w)
    enc = TextPromptEncoder(m)
    g = torch.Generator().manual_seed(T)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).tolist()
    got = enc.encode_ids(ids).float()
    ref = reference_hidden(cfg, w, ids)
    assert got.shape == ref.shape
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 0.03, err
