"""Failure detection of the cross-GPU waits without faulting a GPU.

A bounded barrier waits for a "peer" flag that nothing ever sets (the peer's
flag block is ordinary local memory here).  The wait must give up after its
short limit, set the communication-timeout bit in the status word, and leave
the CUDA context usable.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_times_out_into_status_word():
    from bloom_b200 import ops
    from bloom_b200._ext import cuda

    C = cuda()
    fw = C.tp_flag_words()
    mine = torch.zeros(fw, dtype=torch.int32, device="cuda")
    silent_peer = torch.zeros(fw, dtype=torch.int32, device="cuda")
    st = ops.status()
    st.zero_()
    t0 = time.time()
    C.tp_barrier([mine.data_ptr(), silent_peer.data_ptr()], 0, 0.5, st)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(st[0].item()) & 4, "communication timeout bit not set"
    assert dt < 10
    st.zero_()
    # the context still works
    x = torch.randn(64, 64, device="cuda", dtype=torch.bfloat16)
    y = ops.gemm(x, x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_barrier_single_rank_passes():
    from bloom_b200 import ops
    from bloom_b200._ext import cuda

    C = cuda()
    mine = torch.zeros(C.tp_flag_words(), dtype=torch.int32, device="cuda")
    st = ops.status()
    st.zero_()
    for _ in range(3):
        C.tp_barrier([mine.data_ptr()], 0, 0.5, st)
    torch.cuda.synchronize()
    assert int(st[0].item()) == 0
    assert int(mine[16].item()) == 3  # epoch advanced once per launch
