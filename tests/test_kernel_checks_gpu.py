"""The index-checked kernel build (bloom_b200._C_checked, -DBLOOM_KERNEL_CHECKS).

Each case runs in a child process with BLOOM_KERNEL_CHECKS=1.  An index is
made "out of range" by handing the kernel a view that is smaller than the
allocation behind it: the check must flag the index (status bit 64) and skip
the access, and even a missed check would only touch memory that exists, so
no case can fault the GPU.  A tiny end-to-end generation must also give the
same tokens as the regular build with no bit set.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import json, os, sys
sys.path.insert(0, os.environ["BLOOM_ROOT"])
import torch
from bloom_b200 import ops
from bloom_b200._ext import cuda
C = cuda()
assert C.KERNEL_CHECKS, "the checked build was not loaded"
BIT = C.STATUS_INDEX_CHECK
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
st = ops.status(0)
res = {}

def bits():
    torch.cuda.synchronize()
    v = int(st[0].item())
    st.zero_()
    return v

# embedding: a 64-row table seen as 32 rows; id 40 exists in memory but not in the view
table = torch.randn(64, 128, device=dev).to(torch.bfloat16)
out = ops.embedding(torch.tensor([1, 5], dtype=torch.int32, device=dev), table[:32])
res["embed_ok"] = bits()
out = ops.embedding(torch.tensor([1, 40], dtype=torch.int32, device=dev), table[:32])
res["embed_bad"] = bits()
res["embed_zero_row"] = bool((out[1].float() == 0).all().item())

# rope + KV write: an 8-block cache seen as 4 blocks; slot 100 (block 6) is outside the view
nq, nkv, D = 4, 2, 128
cache = torch.zeros(1, 8, 2, nkv, 16, D, device=dev, dtype=torch.bfloat16)
qkv = torch.randn(2, (nq + 2 * nkv) * D, device=dev).to(torch.bfloat16)
pos = torch.tensor([0, 1], dtype=torch.int64, device=dev)
cs = ops.rope_cos_sin(64, D, 10000.0, device=dev)
q_out = torch.empty(2, nq, D, device=dev, dtype=torch.bfloat16)
ops.rope_kv_write(qkv, pos, torch.tensor([3, 17], dtype=torch.int32, device=dev), cs, q_out, cache[:, :4], 0, nq, nkv)
res["rope_ok"] = bits()
ops.rope_kv_write(qkv, pos, torch.tensor([3, 100], dtype=torch.int32, device=dev), cs, q_out, cache[:, :4], 0, nq, nkv)
res["rope_bad"] = bits()
res["rope_block6_untouched"] = bool((cache[0, 6].float() == 0).all().item())

# decode attention: block id 7 is outside a 4-block view of the cache
cache.normal_()
q = torch.randn(1, 2 * nkv, D, device=dev).to(torch.bfloat16)
o = torch.empty_like(q)
lens = torch.tensor([32], dtype=torch.int32, device=dev)
ops.paged_decode_attention(q, cache[:, :4], 0, torch.tensor([[0, 1]], dtype=torch.int32, device=dev), lens, o,
                           scale=D ** -0.5)
res["decode_ok"] = bits()
ops.paged_decode_attention(q, cache[:, :4], 0, torch.tensor([[0, 7]], dtype=torch.int32, device=dev), lens, o,
                           scale=D ** -0.5)
res["decode_bad"] = bits()

# prefill attention (tcgen05): same out-of-view block id
qp = torch.randn(32, 2 * nkv, D, device=dev).to(torch.bfloat16)
op = torch.empty_like(qp)
cu = torch.tensor([0, 32], dtype=torch.int32, device=dev)
ts, tst = [t.to(dev) for t in ops.prefill_tiles([0, 32], [32])]
for name, bt in (("prefill_ok", [[0, 1]]), ("prefill_bad", [[7, 1]])):
    ops.paged_prefill_attention(qp, cache[:, :4], 0, torch.tensor(bt, dtype=torch.int32, device=dev), lens, cu, ts,
                                tst, op, scale=D ** -0.5)
    res[name] = bits()

# MoE gather / combine: expert rows past the view of the gathered buffer
H, T, K, El = 64, 2, 2, 2
x = torch.randn(T, H, device=dev).to(torch.bfloat16)
ids = torch.tensor([[0, 1], [1, 0]], dtype=torch.int32, device=dev)
slot = torch.tensor([[0, 0], [1, 1]], dtype=torch.int32, device=dev)
posb = torch.empty(T, K, dtype=torch.int32, device=dev)
xs_full = torch.zeros(16, H, device=dev, dtype=torch.bfloat16)
C.moe_gather(x, 0, El, ids, slot, torch.tensor([0, 2], dtype=torch.int32, device=dev), posb, xs_full[:4])
res["moe_ok"] = bits()
C.moe_gather(x, 0, El, ids, slot, torch.tensor([0, 9], dtype=torch.int32, device=dev), posb, xs_full[:4])
res["moe_bad"] = bits()
res["moe_rows_skipped"] = bool((xs_full[9:].float() == 0).all().item()) and int((posb < 0).sum().item()) == 2
ys = torch.randn(16, H, device=dev).to(torch.bfloat16)
outm = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
C.moe_combine(ys[:4], torch.tensor([[0, 1], [2, 9]], dtype=torch.int32, device=dev),
              torch.full((T, K), 0.5, device=dev), outm)
res["combine_bad"] = bits()

# end to end on the tiny model: no bit, tokens printed for comparison with the regular build
from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
from bloom_b200.models.config import preset
from bloom_b200.models.llama import DecoderLM
model = DecoderLM(preset("tiny-llama"), None, dev)
model.random_init(seed=4, std=0.08)
eng = LLMEngine(model, EngineConfig(max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256, num_blocks=32,
                                    use_cuda_graphs=False, autotune=False))
outs = eng.generate([[5, 6, 7, 8, 9], list(range(3, 40))], SamplingParams(max_tokens=6, temperature=0.0,
                                                                          ignore_eos=True))
res["e2e_bits"] = bits()
res["tokens"] = [o.token_ids for o in outs]
res["bit"] = BIT
print(json.dumps(res))
'''


def _regular_tokens():
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM

    dev = torch.device("cuda", 0)
    model = DecoderLM(preset("tiny-llama"), None, dev)
    model.random_init(seed=4, std=0.08)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256, num_blocks=32,
                                        use_cuda_graphs=False, autotune=False))
    outs = eng.generate([[5, 6, 7, 8, 9], list(range(3, 40))], SamplingParams(max_tokens=6, temperature=0.0,
                                                                              ignore_eos=True))
    return [o.token_ids for o in outs]


def test_checked_build_flags_out_of_range_indices():
    if not os.path.exists(os.path.join(ROOT, "bloom_b200")) or not any(
            f.startswith("_C_checked") for f in os.listdir(os.path.join(ROOT, "bloom_b200"))):
        pytest.fail("bloom_b200._C_checked is not built (BLOOM_BUILD=checked python setup.py build_ext --inplace "
                    "--build-temp build/temp_checked)")
    env = dict(os.environ, BLOOM_KERNEL_CHECKS="1", BLOOM_ROOT=ROOT)
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    bit = res["bit"]
    for k in ("embed_ok", "rope_ok", "decode_ok", "prefill_ok", "moe_ok", "e2e_bits"):
        assert res[k] == 0, (k, res)
    for k in ("embed_bad", "rope_bad", "decode_bad", "prefill_bad", "moe_bad", "combine_bad"):
        assert res[k] & bit, (k, res)
    assert res["embed_zero_row"] and res["rope_block6_untouched"] and res["moe_rows_skipped"], res
    assert res["tokens"] == _regular_tokens(), res
