"""Wan VAE decoder on the GPU against the fp32 oracle (random weights, real
channel widths, a 2-frame 4 x 6 latent -> 32 x 48 frames)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vae_decode_matches_oracle():
    from bloom_b200.models.wan_vae import (WanVAE, frames_to_rgb, vae_decode_reference, vae_preset,
                                           vae_random_weights)

    cfg = vae_preset("tiny")
    w = vae_random_weights(cfg, seed=3, device="cuda")
    vae = WanVAE(cfg, "cuda")
    vae.load(w)
    g = torch.Generator(device="cuda").manual_seed(0)
    lat = torch.randn(cfg.latent_channels, 2, 4, 6, device="cuda", generator=g)
    ref = vae_decode_reference(cfg, w, lat)  # [F, 3, 32, 48]
    out = vae.decode(lat, rgb=False).float().permute(0, 3, 1, 2)
    torch.cuda.synchronize()
    assert out.shape == ref.shape
    err = ((out - ref).norm() / ref.norm()).item()
    assert err < 3e-2, err
    rgb = vae.decode(lat)
    torch.cuda.synchronize()
    assert rgb.dtype == torch.uint8 and rgb.shape == (2, 32, 48, 3)
    diff = (rgb.int() - frames_to_rgb(ref).int()).abs().float()
    assert diff.mean().item() < 2.0, diff.mean().item()
    # chunked decoding (one frame at a time) gives the same frames up to accumulation order
    # (GEMM tiling and the GroupNorm partial sums depend on the chunk size)
    vae.max_im2col_bytes = 1
    rgb1 = vae.decode(lat)
    torch.cuda.synchronize()
    d1 = (rgb1.int() - rgb.int()).abs()
    # (one level of rounding at most; the GEMMs pick split-K by the chunk's row count)
    assert d1.max().item() <= 2 and d1.float().mean().item() < 0.25, (d1.max().item(), d1.float().mean().item())
