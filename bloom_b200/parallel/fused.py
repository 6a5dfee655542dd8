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
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops
from .._ext import cuda as _C


class FusedComm:
    def __init__(self, rank: int, world: int, device: torch.device, group=None, max_tokens: int = 8192,
                 hidden: int = 4096, timeout_s: float = 5.0, extra_rows: int = 0):
        import torch.distributed._symmetric_memory as symm

        self.rank, self.world, self.device = rank, world, device
        self.group = group if group is not None else dist.group.WORLD
        self.timeout_s = timeout_s
        self.max_tokens = max_tokens
        self.hidden = hidden
        n = max_tokens * hidden
        # pushed partials use [world][ceil(T / world)][H] slots: up to world - 1 rows more than T
        self._P = symm.empty(n + world * hidden, dtype=torch.bfloat16, device=device)
        self._X = symm.empty(n, dtype=torch.bfloat16, device=device)
        fw = int(_C().tp_flag_words())
        self._F = symm.empty(fw, dtype=torch.int32, device=device)
        self._F.zero_()
        torch.cuda.synchronize(device)
        hP = symm.rendezvous(self._P, self.group)
        hX = symm.rendezvous(self._X, self.group)
        hF = symm.rendezvous(self._F, self.group)
        self._handles = (hP, hX, hF)
        self.p_ptrs = [hP.get_buffer(r, (n + world * hidden,), torch.bfloat16, 0).data_ptr() for r in range(world)]
        self.x_ptrs = [hX.get_buffer(r, (n,), torch.bfloat16, 0).data_ptr() for r in range(world)]
        self.f_ptrs = [hF.get_buffer(r, (fw,), torch.int32, 0).data_ptr() for r in range(world)]
        dist.barrier(group=self.group)

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
                          pushed: bool = False) -> torch.Tensor:
        _C().tp_allreduce_rmsnorm(self.p_ptrs, self.x_ptrs, self.f_ptrs, self.rank, residual, w, eps, T,
                                  self.timeout_s, ops.status(self.device.index), pushed)
        ops._count()
        return self.x(T)

    def barrier(self) -> None:
        _C().tp_barrier(self.f_ptrs, self.rank, self.timeout_s, ops.status(self.device.index))
