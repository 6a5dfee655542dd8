"""int8 KV cache layout helpers (CPU): the reference dequantiser inverts a
hand-built block, and block sizes follow 2 x KVH x 16 x (128 + 4)."""
import pytest
import torch

from bloom_b200 import ops
from bloom_b200.ops.reference import dequant_q8_cache, q8_perm16, quantize_q8_rows


def test_block_bytes_and_head_dim_limit():
    assert ops.kv_q8_block_bytes(8) == 2 * 8 * 16 * 132
    assert ops.kv_q8_block_bytes(1) == 4224
    with pytest.raises(ValueError):
        ops.kv_q8_block_bytes(8, 64)


def test_fragment_order_is_a_permutation_of_each_group():
    assert sorted(q8_perm16(i) for i in range(128)) == list(range(128))
    # thread t of a quad finds elements 2t, 2t+1, 2t+8, 2t+9 at bytes 4t .. 4t+3
    for t in range(4):
        assert [q8_perm16(e) for e in (2 * t, 2 * t + 1, 2 * t + 8, 2 * t + 9)] == [4 * t + j for j in range(4)]


def test_reference_dequantiser_inverts_a_built_block():
    torch.manual_seed(0)
    L, NB, nkv, D = 2, 3, 2, 128
    k = torch.randn(L, NB, nkv, 16, D)
    v = torch.randn(L, NB, nkv, 16, D)
    kq, ks = quantize_q8_rows(k)
    vq, vs = quantize_q8_rows(v)
    P = nkv * 16 * D
    inv_t = torch.empty(16, dtype=torch.long)
    inv_t[torch.tensor([q8_perm16(t) for t in range(16)])] = torch.arange(16)
    buf = torch.zeros(L, NB, ops.kv_q8_block_bytes(nkv), dtype=torch.uint8)
    buf[:, :, :P] = kq.contiguous().to(torch.int8).view(L, NB, -1).view(torch.uint8)
    vt = vq.transpose(-1, -2)[..., inv_t].contiguous()
    buf[:, :, P:2 * P] = vt.to(torch.int8).view(L, NB, -1).view(torch.uint8)
    buf[:, :, 2 * P:] = torch.stack([ks, vs], 2).contiguous().view(L, NB, -1).view(torch.uint8)
    deq = dequant_q8_cache(buf, nkv, D)
    assert deq.shape == (L, NB, 2, nkv, 16, D)
    # int8 rounding: at most half a step (absmax / 254) per element
    assert ((deq[:, :, 0] - k).abs() <= ks[..., None] * 0.5 + 1e-6).all()
    assert ((deq[:, :, 1] - v).abs() <= vs[..., None] * 0.5 + 1e-6).all()


def test_engine_config_reads_kv_dtype(monkeypatch):
    from bloom_b200.engine.engine import EngineConfig

    assert EngineConfig().kv_cache_dtype in ("bf16", "int8")
    monkeypatch.setenv("BLOOM_KV_CACHE_DTYPE", "int8")
    assert EngineConfig().kv_cache_dtype == "int8"
