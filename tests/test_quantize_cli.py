"""bloom_quantize CLI and the C++ quantisers (error bounds, output names)."""
import os

import torch

from bloom_b200.cli.quantize import main
from bloom_b200.formats.safetensors_io import load_file, save_file


def test_quantisers_error_bounds():
    from bloom_b200._ext import runtime

    rt = runtime()
    torch.manual_seed(0)
    w = torch.randn(64, 256) * 0.05
    q, s = rt.quantize_rtn_int8(w)
    assert q.dtype == torch.uint8 and s.shape == (64, 1)
    e8 = (rt.dequant_rtn_int8(q, s) - w).abs().max() / w.abs().max()
    assert e8 < 1 / 127 + 1e-6
    q4, s4, z4 = rt.quantize_rtn_int4(w, 128)
    assert int(q4.max()) <= 15 and s4.shape == (64, 2)
    d4 = rt.dequant_int4(q4, s4, z4, 128)
    assert ((d4 - w).abs() <= s4.repeat_interleave(128, 1) / 2 + 1e-6).all()  # half a step per group
    qa, sa, za, ca = rt.quantize_awq_int4(w, 128)
    da = rt.dequant_int4(qa, sa, za, 128, ca)
    assert ((da - w).norm() / w.norm()).item() < 0.12


def test_cli_roundtrip(tmp_path):
    torch.manual_seed(1)
    sd = {"model.layers.0.mlp.down_proj.weight": torch.randn(32, 256), "model.norm.weight": torch.ones(32),
          "model.layers.0.self_attn.q_norm.weight": torch.ones(16, 8)}
    src = tmp_path / "model.safetensors"
    save_file(sd, str(src))
    for method in ("rtn_int8", "rtn_int4", "awq_int4"):
        dst = tmp_path / f"{method}.safetensors"
        assert main(["-i", str(src), "-o", str(dst), "-m", method, "-g", "64"]) == 0
        out = load_file(str(dst))
        assert "model.layers.0.mlp.down_proj.weight.qweight" in out
        assert "model.norm.weight" in out and "model.layers.0.self_attn.q_norm.weight" in out
        assert ("model.layers.0.mlp.down_proj.weight.zeros" in out) == (method != "rtn_int8")
    assert main(["-i", str(tmp_path / "missing"), "-o", str(tmp_path / "x")]) == 1
