"""The allocation-free decode-attention entry point, called through its C symbol.

bloom_paged_decode_attention_noalloc exists for callers that cannot allocate
GPU memory when they call it (a fixed memory budget set at start-up, a stream
whose pool belongs to another framework, or a C program without PyTorch's
allocator).  It keeps its split-K scratch in a fixed array inside the library.
This test calls it twice in a row and checks each result against the regular
entry point (paged_decode_attention), within the tolerance the other attention
tests use.  This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -2


def _entry_points():
    import bloom_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.bloom_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, ctypes.c_void_p]
    st = lib.bloom_noalloc_status
    st.restype = ctypes.c_int
    st.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return f, st


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


def test_noalloc_decode_attention_matches_regular_entry_point():
    from bloom_b200 import ops

    f, status = _entry_points()
    torch.manual_seed(5)
    L, NB, nq, nkv, D, MB = 2, 400, 32, 8, 128, 80
    cache = torch.randn(L, NB, 2, nkv, 16, D, device="cuda", dtype=torch.bfloat16)
    lens = [3, 40, 333, 900, 1270, 17]
    B = len(lens)
    bt = torch.zeros(B, MB, dtype=torch.int32)
    perm = torch.randperm(NB)
    k = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        bt[b, :n] = perm[k:k + n]
        k += n
    bt = bt.cuda()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, nq, D, device="cuda", dtype=torch.bfloat16)
    layer, splits, scale = 1, 4, 1.0 / math.sqrt(D)
    expected = torch.empty_like(q)
    ops.paged_decode_attention(q, cache, layer, bt, sl, expected, splits=splits, scale=scale)
    stream = torch.cuda.current_stream().cuda_stream
    kv_layer = cache[layer]
    outs = []
    for _ in range(2):  # two calls in a row share (and reuse) the library's scratch array
        out = torch.full_like(q, float("nan"))
        rc = f(q.data_ptr(), out.data_ptr(), kv_layer.data_ptr(), NB, nq, nkv, bt.data_ptr(), bt.stride(0),
               sl.data_ptr(), B, 1, splits, scale, stream)
        assert rc == 0
        outs.append(out)
    torch.cuda.synchronize()
    for out in outs:
        assert torch.isfinite(out.float()).all()
        assert _rel(out, expected) < 2e-2
    bits = ctypes.c_int(-1)
    assert status(ctypes.byref(bits)) == 0 and bits.value == 0


def test_noalloc_rejects_requests_beyond_its_scratch():
    f, _ = _entry_points()
    q = torch.zeros(1, 32, 128, device="cuda", dtype=torch.bfloat16)
    cache = torch.zeros(1, 4, 2, 8, 16, 128, device="cuda", dtype=torch.bfloat16)
    bt = torch.zeros(4096, 4, dtype=torch.int32, device="cuda")
    sl = torch.ones(4096, dtype=torch.int32, device="cuda")
    # 4096 sequences x 8 KV heads x 64 splits x 32 x 130 floats is far beyond the 8 MiB array
    rc = f(q.data_ptr(), q.data_ptr(), cache.data_ptr(), 4, 32, 8, bt.data_ptr(), 4, sl.data_ptr(), 4096, 1, 64,
           1.0, torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
