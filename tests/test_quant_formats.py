"""Quantisation metadata and the fp32 restatements of the AWQ / GPTQ /
bitsandbytes / 8-bit-KV formats (golden values from the reference's tests:
executor/metal_quant.rs:390-425, core/quantization.rs:575-770)."""
import pytest
import torch

from bloom_b200.formats.quant_config import KvCacheDtype, QuantizationConfig, QuantMethod, dequantize_checkpoint
from bloom_b200.ops import reference as R


def test_quant_method_properties_and_hf_aliases():
    assert QuantMethod.AWQ.is_sub_byte() and QuantMethod.GGUF.is_sub_byte() and QuantMethod.FP4.is_sub_byte()
    assert not QuantMethod.NONE.is_sub_byte() and not QuantMethod.FP8.is_sub_byte()
    assert QuantMethod.AWQ.label == "awq" and QuantMethod.HQQ.label == "hqq"
    assert QuantMethod.from_hf_quant_config({"quant_method": "awq", "bits": 4}) == QuantMethod.AWQ
    assert QuantMethod.from_hf_quant_config({"quant_method": "gptq_marlin"}) == QuantMethod.GPTQ
    assert QuantMethod.from_hf_quant_config({"quant_method": "fbgemm_fp8"}) == QuantMethod.FP8
    assert QuantMethod.from_hf_quant_config({"quant_method": "bitsandbytes", "load_in_4bit": True,
                                             "bnb_4bit_quant_type": "nf4"}) == QuantMethod.NF4
    assert QuantMethod.from_hf_quant_config({"quant_method": "bnb", "bnb_4bit_compute_dtype": "bf16"}) == \
        QuantMethod.FP4
    assert QuantMethod.from_hf_quant_config({"quant_method": "bitsandbytes"}) == QuantMethod.INT8
    assert QuantMethod.from_hf_quant_config({}) is None
    assert QuantMethod.from_gguf_type("Q4_K_M") == QuantMethod.GGUF
    assert QuantMethod.from_gguf_type("F16") == QuantMethod.NONE


def test_quantization_config_from_model_config():
    qc = QuantizationConfig.from_model_config({"quantization_config": {"quant_method": "awq", "bits": 4,
                                                                       "group_size": 128}})
    assert qc.weight_method == QuantMethod.AWQ and qc.weight_bits == 4 and qc.group_size == 128
    assert qc.is_quantized() and not qc.has_kv_cache_quant()
    d = QuantizationConfig.from_model_config({})
    assert d.weight_method == QuantMethod.NONE and not d.is_quantized()
    assert QuantizationConfig.from_model_config({"torch_dtype": "bfloat16"}).kv_cache_dtype == KvCacheDtype.BF16
    fp8kv = QuantizationConfig.from_model_config({"quantization_config": {"quant_method": "fp8",
                                                                          "kv_cache_dtype": "fp8"}})
    assert fp8kv.weight_bits == 8 and fp8kv.has_kv_cache_quant()


@pytest.mark.parametrize("name,bits,src", [("Q4_0", 4, "gguf_q4_0"), ("Q8_0", 8, "gguf_q8_0"),
                                           ("IQ2_XXS", 2, "gguf_iq2_xxs"), ("Q4_K_M", 4, "gguf_q4_k_m"),
                                           ("Q6_K", 6, "gguf_q6_k"), ("Q2_K", 2, "gguf_q2_k"),
                                           ("Q5_K_M", 5, "gguf_q5_k_m")])
def test_gguf_quantization_detection(name, bits, src):
    qc = QuantizationConfig.from_gguf_metadata(name)
    assert qc.weight_method == QuantMethod.GGUF and qc.weight_bits == bits and qc.source_format == src
    assert not QuantizationConfig.from_gguf_metadata(None).is_quantized()


def test_kv_dtype_and_memory_ratio():
    assert KvCacheDtype.F16.element_size() == 2 and KvCacheDtype.INT8.element_size() == 1
    assert KvCacheDtype.FP8.needs_dequant() and not KvCacheDtype.F16.needs_dequant()
    qc = QuantizationConfig()
    assert qc.memory_ratio() == 1.0
    qc.weight_bits = 4
    assert qc.memory_ratio() == 0.25


def test_int4_flat_golden_values():
    qw = torch.tensor([0x12345678] * 16, dtype=torch.int32)
    awq = R.dequant_int4_flat(qw, torch.tensor([2.0]), torch.tensor([3], dtype=torch.int32), 128)
    assert awq.shape == (128,) and abs(awq[0] - 10.0) < 1e-3 and abs(awq[1] - 8.0) < 1e-3
    gptq = R.dequant_int4_flat(qw, torch.tensor([2.0, 2.0]), torch.tensor([0x33], dtype=torch.int32), 128,
                               g_idx=torch.zeros(128, dtype=torch.int32))
    assert abs(gptq[0] - 10.0) < 1e-3 and abs(gptq[1] - 8.0) < 1e-3
    # words past the end give 0, as in the reference
    short = R.dequant_int4_flat(qw[:1], torch.tensor([2.0]), torch.tensor([3], dtype=torch.int32), 16)
    assert (short[8:] == 0).all()


def test_nf4_fp4_golden_values():
    packed = torch.tensor([23, 240], dtype=torch.uint8)
    nf4 = R.dequant_bnb4(packed, torch.tensor([2.0]), 4, nf4=True)
    assert torch.allclose(nf4, torch.tensor([-1.3923834, 0.0, 2.0, -2.0]), atol=1e-5)
    fp4 = R.dequant_bnb4(packed, torch.tensor([2.0]), 4, nf4=False)
    assert torch.allclose(fp4, torch.tensor([0.125, 6.0, -6.0, 0.0]), atol=1e-5)


def test_int8_kv_roundtrip():
    x = torch.tensor([[0.5, -0.3, 1.0, -1.0], [0.0, 0.1, -0.7, 0.9]])
    q, s = R.kv_quantize_int8(x)
    assert q.dtype == torch.int8 and s.shape == (2,)
    assert (R.kv_dequantize_int8(q, s) - x).abs().max() < 0.02
    z, zs = R.kv_quantize_int8(torch.zeros(3, 8))
    assert (zs == 1.0).all() and (z == 0).all()


def _to_i32(t):
    return torch.where(t >= 2 ** 31, t - 2 ** 32, t).to(torch.int32)


def pack_gptq(q, z, K, N):
    """Dense codes q [K, N] and zero points z [G, N] -> GPTQ qweight / qzeros (zeros stored minus one)."""
    qw = torch.zeros(K // 8, N, dtype=torch.int64)
    for j in range(8):
        qw |= q[j::8].to(torch.int64) << (4 * j)
    zz = (z - 1).to(torch.int64)
    qz = torch.zeros(z.shape[0], N // 8, dtype=torch.int64)
    for j in range(8):
        qz |= zz[:, j::8] << (4 * j)
    return _to_i32(qw), _to_i32(qz)


def pack_awq(q, z, K, N):
    qw = torch.zeros(K, N // 8, dtype=torch.int64)
    qz = torch.zeros(z.shape[0], N // 8, dtype=torch.int64)
    for j in range(8):
        qw |= q[:, j::8].to(torch.int64) << (4 * R.AWQ_ORDER[j])
        qz |= z[:, j::8].to(torch.int64) << (4 * R.AWQ_ORDER[j])
    return _to_i32(qw), _to_i32(qz)


def test_gptq_awq_checkpoint_conversion():
    torch.manual_seed(0)
    K, N, G = 64, 16, 32
    q = torch.randint(0, 16, (K, N))
    z = torch.randint(1, 16, (K // G, N))
    s = (torch.rand(K // G, N) + 0.5).half()
    g_idx = torch.arange(K) // G
    want = ((q.float() - z[g_idx].float()) * s.float()[g_idx]).t()
    qw, qz = pack_gptq(q, z, K, N)
    assert torch.allclose(R.dequant_gptq(qw, qz, s, g_idx.to(torch.int32)), want, atol=1e-4)
    aw, az = pack_awq(q, z, K, N)
    assert torch.allclose(R.dequant_awq(aw, az, s, G), want, atol=1e-4)
    sd = {"l.qweight": qw, "l.qzeros": qz, "l.scales": s, "l.g_idx": g_idx.to(torch.int32), "n.weight": torch.ones(4)}
    qc = QuantizationConfig.from_model_config({"quantization_config": {"quant_method": "gptq", "bits": 4,
                                                                       "group_size": G}})
    out = dequantize_checkpoint(sd, qc)
    assert set(out) == {"l.weight", "n.weight"} and out["l.weight"].dtype == torch.bfloat16
    assert torch.allclose(out["l.weight"].float(), want, atol=0.1, rtol=0.01)


def test_mrope_cpu_matches_torch_restatement():
    from bloom_b200._ext import runtime

    rt = runtime()
    torch.manual_seed(1)
    B, H, S, D = 2, 3, 5, 128
    x = torch.randn(B, H, S, D)
    pos = torch.randint(0, 50, (3, B, S))
    from bloom_b200 import ops

    cos, sin = ops.mrope_cos_sin(pos, D)
    got = rt.mrope_cpu(x, cos, sin, 24, 20, 20)
    assert torch.allclose(got, R.mrope(x, cos, sin), atol=1e-5)
    # text-only positions (all three planes equal) reduce to ordinary rotate-half RoPE
    p1 = torch.arange(S).expand(3, B, S)
    c1, s1 = ops.mrope_cos_sin(p1, D)
    plain = x * c1[0][:, None] + torch.cat([-x[..., D // 2:], x[..., :D // 2]], -1) * s1[0][:, None]
    assert torch.allclose(rt.mrope_cpu(x, c1, s1, 24, 20, 20), plain, atol=1e-5)


def test_cpu_oracle_kernels():
    from bloom_b200._ext import runtime

    rt = runtime()
    torch.manual_seed(4)
    a, b = torch.randn(1000), torch.randn(1000)
    assert torch.allclose(rt.oracle_vector_add(a, b), a + b)
    A, B = torch.randn(17, 33), torch.randn(33, 9)
    assert torch.allclose(rt.oracle_matmul(A, B), A @ B, atol=1e-4)
    x = torch.randn(257) * 5
    assert torch.allclose(rt.oracle_softmax(x), torch.softmax(x, 0), atol=1e-6)
    q, k, v = torch.randn(3, 40, 64).unbind(0)
    want = torch.softmax(q @ k.t() / 8.0, dim=-1) @ v
    assert torch.allclose(rt.oracle_attention(q, k, v), want, atol=1e-4)
