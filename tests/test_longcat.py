"""LongCat host-side pieces (CPU): latent packing, token positions, RoPE
table, and the fp32 oracles' shapes."""
import math

import torch

from bloom_b200.models.longcat import (klvae_preset, klvae_random_weights, klvae_reference, longcat_preset,
                                       longcat_random_weights, longcat_transformer_reference, pack_latents,
                                       rope_table, token_positions, unpack_latents)


def test_pack_unpack_roundtrip():
    lat = torch.randn(16, 6, 10)
    p = pack_latents(lat)
    assert p.shape == (15, 64)
    assert torch.equal(unpack_latents(p, 16, 6, 10), lat)
    # token (row 1, col 2) holds the 2x2 patch at rows 2-3, cols 4-5, channel-major
    assert torch.equal(p[1 * 5 + 2].view(16, 2, 2), lat[:, 2:4, 4:6])


def test_positions_and_rope_axes():
    pos = token_positions(3, 2, 4)
    assert pos.tolist()[:3] == [[0, 0, 0], [0, 0, 1], [0, 0, 2]]
    assert pos.tolist()[3 + 5] == [0, 1, 1]
    cfg = longcat_preset("tiny-longcat")
    t = rope_table(cfg, 8)
    assert t.shape == (8, 64, 2)
    # first pair of each axis (0, 8, 36) turns one radian per position
    for p in (0, 8, 36):
        assert math.isclose(float(t[2, p, 0]), math.cos(2.0), rel_tol=1e-6)


def test_oracles_shapes():
    cfg = longcat_preset("tiny-longcat")
    w = longcat_random_weights(cfg, seed=0)
    out = longcat_transformer_reference(cfg, w, torch.randn(6, 64), torch.randn(4, cfg.joint_attention_dim), 0.5,
                                        (2, 3))
    assert out.shape == (6, 64) and torch.isfinite(out).all()
    vc = klvae_preset("tiny")
    vw = klvae_random_weights(vc, seed=0)
    lat = klvae_reference(vc, vw, image=torch.rand(3, 16, 32) * 2 - 1)
    assert lat.shape == (16, 8, 16)
    assert klvae_reference(vc, vw, latent=lat).shape == (3, 16, 32)
