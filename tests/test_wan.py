"""Wan 2.1 host-side pieces (CPU): schedule, embeddings, RoPE table, oracle shapes."""
import math

import torch

from bloom_b200.models.wan import (rope_axes, rope_table, sampling_sigmas, sinusoidal, wan_dit_reference, wan_preset,
                                   wan_random_weights)


def test_sampling_sigmas_schedule():
    s = sampling_sigmas(50, 5.0)
    assert len(s) == 51 and s[0] == 1.0 and s[-1] == 0.0
    assert all(a > b for a, b in zip(s, s[1:]))
    assert s[25] > sampling_sigmas(50, 1.0)[25]  # the shift keeps sigma high for longer
    assert sampling_sigmas(4, 1.0) == [1.0, 0.75, 0.5, 0.25, 0.0]


def test_rope_axes_and_table():
    assert rope_axes(128) == (44, 42, 42)
    t = rope_table(128, positions=8)
    assert t.shape == (8, 64, 2)
    assert torch.allclose(t[0, :, 0], torch.ones(64)) and torch.allclose(t[0, :, 1], torch.zeros(64))
    # pair 0 of each axis turns by one radian per position
    for p in (0, 22, 43):
        assert math.isclose(float(t[3, p, 0]), math.cos(3.0), rel_tol=1e-6)


def test_sinusoidal_embedding():
    e = sinusoidal(8, torch.tensor([0.0, 1000.0]))
    assert e.shape == (2, 8)
    assert torch.allclose(e[0], torch.tensor([1.0] * 4 + [0.0] * 4, dtype=torch.float64))
    assert math.isclose(float(e[1, 0]), math.cos(1000.0), rel_tol=1e-9)


def test_oracle_shapes_and_time_dependence():
    cfg = wan_preset("tiny-wan")
    w = wan_random_weights(cfg, seed=0)
    lat = torch.randn(1, cfg.in_dim, 2, 4, 4)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim)
    v1 = wan_dit_reference(cfg, w, lat, torch.tensor([900.0]), ctx)
    v2 = wan_dit_reference(cfg, w, lat, torch.tensor([100.0]), ctx)
    assert v1.shape == lat.shape and torch.isfinite(v1).all()
    assert not torch.allclose(v1, v2)


def test_t5_relative_buckets_and_oracle_padding():
    from bloom_b200.models.umt5 import relative_buckets, t5_encode_reference, t5_preset, t5_random_weights

    b = relative_buckets(torch.arange(-3, 4)).tolist()
    assert b == [3, 2, 1, 0, 17, 18, 19]  # exact near zero, the upper half for keys after the query
    assert relative_buckets(torch.tensor([-1000, 1000])).tolist() == [15, 31]
    cfg = t5_preset("tiny")
    w = t5_random_weights(cfg, seed=1)
    ids = torch.randint(1, cfg.vocab_size, (2, cfg.max_length))
    out = t5_encode_reference(cfg, w, ids, [10, 24])
    assert out.shape == (2, cfg.max_length, cfg.d_model)
    assert (out[0, 10:] == 0).all() and out[0, :10].abs().sum() > 0
    # padding tokens do not change the real positions' outputs
    ids2 = ids.clone()
    ids2[0, 10:] = 0
    assert torch.allclose(t5_encode_reference(cfg, w, ids2, [10, 24])[0, :10], out[0, :10], atol=1e-4)
