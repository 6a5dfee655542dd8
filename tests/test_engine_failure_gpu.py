"""Kernel status errors reach the requests, without faulting a GPU.

One GPU plays rank 0 of a two-rank tensor-parallel engine.  The "peer" is
ordinary local memory that no process services, so the first fused
collective's bounded wait for the peer's ready flag gives up after its short
limit.  That must poison the communicator (later collectives do nothing),
and the status word that comes back with the sampled tokens must make the
engine fail the step's request with finish_reason "error" -- no tokens --
and drop the fused communicator.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _fake_two_rank_fused(dev, T, H, timeout_s):
    """A FusedComm whose peer buffers are local allocations nothing writes to."""
    from bloom_b200._ext import cuda
    from bloom_b200.parallel.fused import FusedComm

    fc = FusedComm.__new__(FusedComm)
    fc.rank, fc.world, fc.device, fc.group = 0, 2, dev, None
    fc.timeout_s, fc.max_tokens, fc.hidden = timeout_s, T, H
    fc.max_logit_rows = T
    fw = int(cuda().tp_flag_words())
    n = T * H
    keep = []

    def buf(numel, dtype):
        t = torch.zeros(numel, dtype=dtype, device=dev)
        keep.append(t)
        return t

    fc._P, peerP = buf(n + 2 * H, torch.bfloat16), buf(n + 2 * H, torch.bfloat16)
    fc._X, peerX = buf(n, torch.bfloat16), buf(n, torch.bfloat16)
    fc._F, peerF = buf(fw, torch.int32), buf(fw, torch.int32)
    ns = 2 * (T + 1) * 2
    fc._G, peerG = buf(ns, torch.int32), buf(ns, torch.int32)
    fc.p_ptrs = [fc._P.data_ptr(), peerP.data_ptr()]
    fc.x_ptrs = [fc._X.data_ptr(), peerX.data_ptr()]
    fc.f_ptrs = [fc._F.data_ptr(), peerF.data_ptr()]
    fc.g_ptrs = [fc._G.data_ptr(), peerG.data_ptr()]
    fc._full = None
    fc._guards = {}
    fc.poisoned = False
    fc._keep = keep
    return fc


def test_comm_timeout_fails_the_request_not_the_gpu():
    from bloom_b200 import ops
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM, TPInfo
    from bloom_b200.parallel.comm import Communicator

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset("tiny-tp")
    comm = Communicator(0, 2, dev, None, mode="nccl")
    comm.fused = _fake_two_rank_fused(dev, 256, cfg.hidden_size, timeout_s=0.3)
    comm.mode = "fused"
    model = DecoderLM(cfg, TPInfo(0, 2, None, comm), dev)
    model.random_init(seed=1)
    ops.status(0).zero_()
    eng = LLMEngine(model, EngineConfig(max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256,
                                        num_blocks=32, use_cuda_graphs=False, autotune=False))
    rid = eng.add_request([5, 6, 7, 8], SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True))
    outs = eng.step()
    torch.cuda.synchronize()
    assert len(outs) == 1 and outs[0].request_id == rid
    r = outs[0]
    assert r.finished and r.finish_reason == "error" and r.token_ids == []
    assert "cross-GPU wait timed out" in r.error
    assert not eng.has_unfinished()
    assert comm.fused is None and comm.mode == "nccl"  # the poisoned communicator was dropped
    assert len(eng.failures) == 1 and eng.failures[0]["status"] & 4
    assert int(ops.status(0)[0].item()) == 0  # cleared for the next step
    # the context still works
    x = torch.randn(64, 64, device=dev, dtype=torch.bfloat16)
    y = ops.gemm(x, x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_poisoned_collective_does_nothing():
    """After one timeout, a second launch returns at once with the poisoned bit."""
    import time

    from bloom_b200 import ops
    from bloom_b200._ext import cuda

    C = cuda()
    fw = C.tp_flag_words()
    mine = torch.zeros(fw, dtype=torch.int32, device="cuda")
    silent_peer = torch.zeros(fw, dtype=torch.int32, device="cuda")
    st = ops.status()
    st.zero_()
    C.tp_barrier([mine.data_ptr(), silent_peer.data_ptr()], 0, 0.3, st)
    torch.cuda.synchronize()
    assert int(st[0].item()) & 4
    assert int(mine[18].item()) == 1  # poison word
    epoch = int(mine[16].item())
    st.zero_()
    t0 = time.time()
    C.tp_barrier([mine.data_ptr(), silent_peer.data_ptr()], 0, 5.0, st)
    torch.cuda.synchronize()
    assert time.time() - t0 < 2.0  # no second wait
    assert int(st[0].item()) == 32
    assert int(mine[16].item()) == epoch  # the epoch no longer advances
    st.zero_()


def test_argmax_gather_single_rank_matches_argmax():
    """The fused logits arg-max + gather at world 1 equals the plain arg-max,
    and its last entry carries the status word."""
    from bloom_b200 import ops
    from bloom_b200._ext import cuda

    C = cuda()
    torch.manual_seed(0)
    NL, V = 37, 16032
    logits = torch.randn(NL, V, device="cuda").to(torch.bfloat16)
    logits[3, 100] = logits[3, 200] = 50.0  # tie: the lower index wins
    flags = torch.zeros(C.tp_flag_words(), dtype=torch.int32, device="cuda")
    slots = torch.zeros(1 * (64 + 1) * 2, dtype=torch.int32, device="cuda")
    out = torch.full((NL + 1,), -7, dtype=torch.int32, device="cuda")
    st = ops.status()
    st.zero_()
    for _ in range(2):
        C.tp_argmax_gather(logits, 1000, [slots.data_ptr()], 64, [flags.data_ptr()], 0, out, 1.0, st)
    torch.cuda.synchronize()
    ref = logits.float().argmax(1).to(torch.int32) + 1000
    assert torch.equal(out[:NL], ref)
    assert int(out[3]) == 1100
    assert int(out[NL]) == 0
    assert int(flags[16].item()) == 2


def test_gather_cols_single_rank_copies_rows():
    from bloom_b200 import ops
    from bloom_b200._ext import cuda

    C = cuda()
    NL, V = 9, 4096
    logits = torch.randn(NL, V + 64, device="cuda").to(torch.bfloat16)[:, :V]
    flags = torch.zeros(C.tp_flag_words(), dtype=torch.int32, device="cuda")
    dst = torch.zeros(NL * V, dtype=torch.bfloat16, device="cuda")
    stat = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_st = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    st = ops.status()
    st.zero_()
    C.tp_gather_cols(logits, [dst.data_ptr()], V, [stat.data_ptr()], [flags.data_ptr()], 0, out_st, 1.0, st)
    torch.cuda.synchronize()
    assert torch.equal(dst.view(NL, V), logits)
    assert int(out_st.item()) == 0
