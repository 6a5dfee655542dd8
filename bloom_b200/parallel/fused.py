"""Fused tensor-parallel collectives over NVLink peer memory.

Buffers are allocated with torch's symmetric memory (cuMem-based mappings of
every rank's allocation into every process: the plumbing); all data movement
and synchronisation is done by this repository's kernels (csrc/kernels/comm.cu)
with 16-byte P2P loads/stores and bounded flag waits.

Per row-parallel GEMM the model calls `allreduce_rmsnorm`.  Dense layers run
the GEMM with `push_args(T)`: its epilogue stores each finished output tile
row straight into the owning rank's buffer over NVLink (the reduce-scatter
is fused into the tcgen05 GEMM and overlaps its remaining tiles), and one
kernel sums the local slots, adds the residual, applies RMSNorm and
all-gathers the result into `x(T)` on every rank, which is the next GEMM's
input.  Other producers (MoE) write `partial(T)` locally and the same kernel
pulls the peers' rows instead.

No kernel here uses an NVLink multicast object, so none is created: torch's
symmetric memory would otherwise bind every rendezvoused buffer to one, and a
rank that dies while bound to it can raise NVLink faults on its peers' GPUs.
`TORCH_SYMM_MEM_DISABLE_MULTICAST=1` is set before the first allocation and
every handle is checked to carry no multicast pointer.

Every symmetric buffer carries a 4 KiB guard region before and after its
data, filled with a fixed word pattern; kernels receive pointers to the data
only.  `check_canaries()` counts guard words that no longer hold the pattern
on this rank (a stray P2P store from any rank lands in some rank's guard),
and the TP tests assert it is zero after every run.
"""
from __future__ import annotations

import os
from typing import List, Optional

os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from .. import ops  # noqa: E402
from .._ext import cuda as _C  # noqa: E402

CANARY_BYTES = 4096
CANARY_WORD = 0x5AC3A55A  # as two bf16 halves: finite values, so a guard never reads as NaN


def _guarded(symm, numel: int, dtype, device):
    """(full symmetric tensor, data view, guard elements) with both guards filled."""
    es = torch.empty(0, dtype=dtype).element_size()
    g = CANARY_BYTES // es
    full = symm.empty(numel + 2 * g, dtype=dtype, device=device)
    words = full.view(torch.int32)
    gw = CANARY_BYTES // 4
    words[:gw].fill_(CANARY_WORD)
    words[words.numel() - gw:].fill_(CANARY_WORD)
    return full, full[g:g + numel], g


def _bad_guard_words(full: torch.Tensor) -> int:
    words = full.view(torch.int32)
    gw = CANARY_BYTES // 4
    return int((words[:gw] != CANARY_WORD).sum().item() + (words[words.numel() - gw:] != CANARY_WORD).sum().item())


def _peer(handle, rank: int, full_numel: int, dtype, guard: int) -> int:
    es = torch.empty(0, dtype=dtype).element_size()
    return handle.get_buffer(rank, (full_numel,), dtype, 0).data_ptr() + guard * es


class FusedComm:
    def __init__(self, rank: int, world: int, device: torch.device, group=None, max_tokens: int = 8192,
                 hidden: int = 4096, timeout_s: float = 5.0, extra_rows: int = 0, max_logit_rows: int = 0):
        import torch.distributed._symmetric_memory as symm

        self.rank, self.world, self.device = rank, world, device
        self.group = group if group is not None else dist.group.WORLD
        self.timeout_s = timeout_s
        self.max_tokens = max_tokens
        self.hidden = hidden
        n = max_tokens * hidden
        # pushed partials use [world][ceil(T / world)][H] slots: up to world - 1 rows more than T
        bf, i32 = torch.bfloat16, torch.int32
        fP, self._P, gP = _guarded(symm, n + world * hidden, bf, device)
        fX, self._X, gX = _guarded(symm, n, bf, device)
        fw = int(_C().tp_flag_words())
        fF, self._F, gF = _guarded(symm, fw, i32, device)
        self._F.zero_()
        # greedy logits: (value, global index) pairs [world][rows + 1] (last entry: a rank's status word)
        self.max_logit_rows = int(max_logit_rows or max_tokens)
        ns = world * (self.max_logit_rows + 1) * 2
        fG, self._G, gG = _guarded(symm, ns, i32, device)
        self._G.zero_()
        self._guards = {"partial": fP, "x": fX, "flags": fF, "logit_pairs": fG}
        torch.cuda.synchronize(device)
        hP = symm.rendezvous(fP, self.group)
        hX = symm.rendezvous(fX, self.group)
        hF = symm.rendezvous(fF, self.group)
        hG = symm.rendezvous(fG, self.group)
        self._handles = (hP, hX, hF, hG)
        self._full = None  # lazily: full-vocabulary logits rows for stochastic sampling
        self.poisoned = False
        for h in self._handles:
            mc = getattr(h, "multicast_ptr", 0)
            if mc:
                raise RuntimeError("symmetric-memory buffer is bound to an NVLink multicast object although "
                                   "TORCH_SYMM_MEM_DISABLE_MULTICAST=1; refusing to run the fused collectives")
        self.g_ptrs = [_peer(hG, r, fG.numel(), i32, gG) for r in range(world)]
        self.p_ptrs = [_peer(hP, r, fP.numel(), bf, gP) for r in range(world)]
        self.x_ptrs = [_peer(hX, r, fX.numel(), bf, gX) for r in range(world)]
        self.f_ptrs = [_peer(hF, r, fF.numel(), i32, gF) for r in range(world)]
        dist.barrier(group=self.group)

    def check_canaries(self) -> dict:
        """Guard words of this rank's symmetric buffers that lost their pattern
        (0 everywhere when no kernel wrote outside a buffer).  Synchronises."""
        torch.cuda.synchronize(self.device)
        return {k: _bad_guard_words(v) for k, v in self._guards.items()}

    def can_all_reduce(self, t: torch.Tensor) -> bool:
        return False  # the fused path is taken through allreduce_rmsnorm, not a bare all-reduce

    def partial(self, T: int) -> torch.Tensor:
        """[T, H] bf16 view of this rank's peer-visible partial-sum buffer (GEMM output)."""
        assert T <= self.max_tokens
        return self._P[:T * self.hidden].view(T, self.hidden)

    def push_args(self, T: int):
        """(peer buffers, this rank, rows per rank) for ops.gemm(push=...): the
        GEMM writes token row t into rank t // rows's buffer, slot [rank][t % rows]."""
        return self.p_ptrs, self.rank, (T + self.world - 1) // self.world

    def x(self, T: int) -> torch.Tensor:
        """[T, H] bf16 view of this rank's all-gathered input buffer."""
        return self._X[:T * self.hidden].view(T, self.hidden)

    def allreduce_rmsnorm(self, T: int, residual: torch.Tensor, w: torch.Tensor, eps: float,
                          pushed: bool = False, defer: bool = False) -> torch.Tensor:
        """defer=True: the kernel does not wait for the peers' rows; the next
        reader of x(T) must be an ops.gemm given wait=self.wait_args(), which
        waits for them before its first activation tile (the wait overlaps the
        collective's exit and the GEMM's weight prefetch)."""
        _C().tp_allreduce_rmsnorm(self.p_ptrs, self.x_ptrs, self.f_ptrs, self.rank, residual, w, eps, T,
                                  self.timeout_s, ops.status(self.device.index), pushed, defer)
        ops._count()
        return self.x(T)

    def wait_args(self):
        """(this rank's flag block, timeout) for ops.gemm(wait=...)."""
        return self.f_ptrs[self.rank], self.timeout_s

    def barrier(self) -> None:
        _C().tp_barrier(self.f_ptrs, self.rank, self.timeout_s, ops.status(self.device.index))

    # ------------------------------------------------------------ last-layer logits
    def argmax_gather(self, logits: torch.Tensor, vocab_offset: int, out: torch.Tensor) -> torch.Tensor:
        """Greedy tokens of vocabulary-parallel logits in one kernel: local
        argmax, (value, index) pairs stored into every rank over NVLink,
        bounded flag exchange, reduction.  out: int32 [NL + 1]; out[NL] is the
        OR of every rank's status word (all ranks read the same value)."""
        _C().tp_argmax_gather(logits, int(vocab_offset), self.g_ptrs, self.max_logit_rows, self.f_ptrs, self.rank,
                              out, self.timeout_s, ops.status(self.device.index))
        ops._count()
        return out

    def gather_cols(self, logits: torch.Tensor, out_status: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary rows [NL, world * Vl] on every rank from the
        [NL, Vl] shards (16-byte P2P stores); out_status[0] receives the OR of
        every rank's status word.  The first call allocates the buffers on all
        ranks at once (the ranks run identical schedules)."""
        import torch.distributed._symmetric_memory as symm

        NL, Vl = logits.shape
        V = Vl * self.world
        if self._full is None or self._full[1] < NL or self._full[2] != V:
            rows = max(NL, self.max_logit_rows)
            fL, L, gL = _guarded(symm, rows * V, torch.bfloat16, self.device)
            fS, S, gS = _guarded(symm, self.world, torch.int32, self.device)
            S.zero_()
            self._guards["logit_rows"], self._guards["logit_status"] = fL, fS
            torch.cuda.synchronize(self.device)
            hL = symm.rendezvous(fL, self.group)
            hS = symm.rendezvous(fS, self.group)
            for h in (hL, hS):
                if getattr(h, "multicast_ptr", 0):
                    raise RuntimeError("symmetric-memory buffer is bound to an NVLink multicast object")
            lp = [_peer(hL, r, fL.numel(), torch.bfloat16, gL) for r in range(self.world)]
            sp = [_peer(hS, r, fS.numel(), torch.int32, gS) for r in range(self.world)]
            self._full = (L, rows, V, lp, sp, (hL, hS))
        L, rows, V, lp, sp, _ = self._full
        _C().tp_gather_cols(logits.contiguous(), lp, V, sp, self.f_ptrs, self.rank, out_status, self.timeout_s,
                            ops.status(self.device.index))
        ops._count()
        return L[:NL * V].view(NL, V)
