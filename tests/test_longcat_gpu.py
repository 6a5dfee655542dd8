"""LongCat image edit on the GPU against fp32 oracles (random weights, tiny
shapes with the real head dim and RoPE axes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_longcat_transformer_matches_oracle():
    from bloom_b200.models.longcat import (LongCatTransformer, longcat_preset, longcat_random_weights,
                                           longcat_transformer_reference)

    cfg = longcat_preset("tiny-longcat")
    w = longcat_random_weights(cfg, seed=1, device="cuda")
    tr = LongCatTransformer(cfg, "cuda")
    tr.load(w)
    g = torch.Generator(device="cuda").manual_seed(1)
    for Lt, grid in ((5, (3, 4)), (40, (6, 10))):  # 17 and 100 joint tokens (one / several pages, two tiles)
        packed = torch.randn(grid[0] * grid[1], cfg.in_channels, device="cuda", generator=g).to(torch.bfloat16)
        ctx = torch.randn(Lt, cfg.joint_attention_dim, device="cuda", generator=g).to(torch.bfloat16)
        out = tr.forward(packed, ctx, 0.5, grid).float()
        torch.cuda.synchronize()
        ref = longcat_transformer_reference(cfg, w, packed, ctx, 0.5, grid)
        err = ((out - ref).norm() / ref.norm()).item()
        assert err < 3e-2, (Lt, grid, err)


def test_kl_vae_encode_decode_match_oracle():
    from bloom_b200.models.longcat import KLVae, klvae_preset, klvae_random_weights, klvae_reference

    cfg = klvae_preset("tiny")
    w = klvae_random_weights(cfg, seed=2, device="cuda")
    vae = KLVae(cfg, "cuda")
    vae.load(w)
    g = torch.Generator(device="cuda").manual_seed(2)
    img = torch.rand(3, 32, 48, device="cuda", generator=g) * 2 - 1
    lat = vae.encode(img)
    torch.cuda.synchronize()
    ref = klvae_reference(cfg, w, image=img)
    assert lat.shape == ref.shape == (16, 16, 24)
    assert ((lat - ref).norm() / ref.norm()).item() < 3e-2
    dec = vae.decode_image(ref, rgb=False).float().permute(2, 0, 1)
    torch.cuda.synchronize()
    dref = klvae_reference(cfg, w, latent=ref)
    assert dec.shape == dref.shape == (3, 32, 48)
    assert ((dec - dref).norm() / dref.norm()).item() < 3e-2


def test_longcat_draft_edit_pipeline():
    from bloom_b200.models.longcat import LongCatEditPipeline

    pipe = LongCatEditPipeline.from_presets("tiny-longcat", "tiny", seed=0, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    img = torch.randint(0, 256, (32, 48, 3), device="cuda", generator=g, dtype=torch.uint8)
    emb = torch.randn(7, pipe.tr.cfg.joint_attention_dim, device="cuda", generator=g)
    out = pipe.edit(img, emb)
    torch.cuda.synchronize()
    assert out.shape == (32, 48, 3) and out.dtype == torch.uint8
    # strength 0 reproduces the VAE round trip of the input
    pipe.strength = 0.0
    base = pipe.edit(img, emb)
    torch.cuda.synchronize()
    assert not torch.equal(out, base)
