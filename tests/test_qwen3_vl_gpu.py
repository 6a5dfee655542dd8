"""Qwen3-VL on the GPU kernels vs the fp32 PyTorch oracle: vision tower
tokens and deepstack features, greedy generation with an image and text-only."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup():
    from bloom_b200.engine.processor import qwen_vl_patches
    from bloom_b200.models.qwen3_vl import Qwen3VL, vl_preset

    cfg = vl_preset("tiny-qwen3-vl")
    w = Qwen3VL.random_weights(cfg, seed=0)
    m = Qwen3VL(cfg, "cuda")
    m.load(w)
    img = np.random.default_rng(1).integers(0, 256, (64, 96, 3), dtype=np.uint8)
    patches, grid = qwen_vl_patches(img, cfg.vision, min_pixels=1, max_pixels=10 ** 6)
    return cfg, w, m, patches, grid


def _rel(a, b):
    return (a.float().cpu() - b.float()).norm().item() / max(1e-6, b.float().norm().item())


def test_vision_tower_matches_oracle():
    from bloom_b200.models.qwen3_vl import reference_vision

    cfg, w, m, patches, grid = _setup()
    toks, feats = m.encode_image(patches, grid)
    rt, rf = reference_vision(cfg, w, patches, grid)
    assert toks.shape == rt.shape == (grid[1] * grid[2] // 4, cfg.vision.out_hidden_size)
    assert _rel(toks, rt) < 3e-2, _rel(toks, rt)
    assert len(feats) == len(rf) == 2 and all(_rel(a, b) < 3e-2 for a, b in zip(feats, rf))


@pytest.mark.parametrize("with_image", [True, False])
def test_generation_matches_oracle(with_image):
    from bloom_b200.models.qwen3_vl import reference_logits

    cfg, w, m, patches, grid = _setup()
    n = grid[1] * grid[2] // 4
    ids = m.prompt_ids([5, 6, 7], n if with_image else 0, prefix=[11, 12])
    out = m.generate(ids, patches if with_image else None, grid if with_image else None, max_tokens=8)
    assert len(out) == 8
    logits = reference_logits(cfg, w, ids + out[:-1], patches if with_image else None, grid if with_image else None)
    for j, tok in enumerate(out):
        row = logits[len(ids) - 1 + j]
        spread = (row.max() - row.median()).item()
        gap = (row.max() - row[tok]).item()
        assert gap <= 0.05 * spread + 1e-4, (j, tok, gap, spread)
    from bloom_b200 import ops

    assert int(ops.status()[0].item()) == 0
