"""Tensor-parallel communicator.

Process model: one process per GPU, `torch.distributed` (backend "nccl") for
rendezvous and as the baseline collective path.  Replaces the reference's
no-op `CollectiveOps` / `TensorCollectiveOps` (crates/engine/src/core/
parallelism.rs:105-178), which never moved a byte between devices.

Modes
  nccl   baseline: row-parallel outputs are summed with NCCL all-reduce,
         logits are reduced with a distributed arg-max (8 bytes per row per
         rank) or all-gathered for stochastic sampling.
  fused  the peer-memory kernels in bloom_b200.parallel.fused (GEMM epilogue
         writes straight into peers' buffers over NVLink; the logits arg-max
         and its all-gather are one kernel), with NCCL kept for bootstrap.

Every sampling call returns int32 [NL + 1]: the tokens and, in the last
entry, the OR of all ranks' kernel status words, so every rank sees the same
error bits after a step and fails the same requests.  When those bits say
the fused communicator timed out (or is poisoned), `poison()` drops it and
the communicator continues on NCCL.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


class Communicator:
    def __init__(self, rank: int, size: int, device: torch.device, group=None, mode: str = "nccl",
                 max_tokens: int = 8192, hidden: int = 4096, timeout_s: float = 5.0):
        self.rank = rank
        self.size = size
        self.device = device
        self.group = group
        self.mode = mode
        self.fused = None
        if mode == "fused" and size > 1:
            from .fused import FusedComm

            self.fused = FusedComm(rank, size, device, group, max_tokens=max_tokens, hidden=hidden,
                                   timeout_s=timeout_s)

    # ------------------------------------------------------------ collectives
    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        if self.fused is not None and self.fused.can_all_reduce(t):
            return self.fused.all_reduce(t)
        dist.all_reduce(t, group=self.group)
        return t

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        out = torch.empty((self.size,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.group)

    # ------------------------------------------------------------ failure handling
    COMM_BITS = 4 | 32  # cross-GPU wait timed out | communicator poisoned

    def poison(self) -> bool:
        """Stop using the fused communicator after a timeout (every live rank
        sees the same bits in the same step and calls this together); later
        collectives run on NCCL.  Returns True if the mode changed."""
        if self.fused is None:
            return False
        self.fused.poisoned = True
        self.fused = None
        self.mode = "nccl"
        return True

    # ------------------------------------------------------------ sampling over a vocab-parallel lm_head
    def sample_vocab_parallel(self, logits: torch.Tensor, greedy: bool, sampling, vocab_local: int) -> torch.Tensor:
        """Tokens of every logits row plus the ranks' combined status: int32 [NL + 1]."""
        NL = logits.shape[0]
        out = torch.empty(NL + 1, dtype=torch.int32, device=logits.device)
        st = ops.status(self.device.index)
        if self.fused is not None and NL <= self.fused.max_logit_rows:
            if greedy:
                return self.fused.argmax_gather(logits, self.rank * vocab_local, out)
            full = self.fused.gather_cols(logits, out[NL:])
            ops.sample(full, *sampling, out=out[:NL])
            return out
        if greedy:
            idx = ops.argmax(logits)
            val = logits.gather(1, idx.long().unsqueeze(1)).float().squeeze(1)
            gidx = (idx.long() + self.rank * vocab_local).float()
            pack = torch.stack([val, gidx], 1)  # [NL, 2] f32 (indices < 2^24 are exact)
            pack = torch.cat([pack, torch.stack([st[:1].float(), st[:1].float()], 1)], 0)  # + status row
            allp = self.all_gather_rows(pack)  # [size, NL + 1, 2]
            best = allp[:, :NL, 0].argmax(0)  # first rank wins ties -> lowest global index
            out[:NL] = allp[:, :NL].gather(0, best.view(1, NL, 1).expand(1, NL, 2))[0, :, 1].to(torch.int32)
            out[NL:] = _or_reduce(allp[:, NL, 0].to(torch.int32))
            return out
        full = self.all_gather_rows(logits)  # [size, NL, Vl]
        full = full.permute(1, 0, 2).reshape(NL, self.size * vocab_local).contiguous()
        ops.sample(full, *sampling, out=out[:NL])
        out[NL:] = _or_reduce(self.all_gather_rows(st[:1].clone()).view(-1))
        return out


def _or_reduce(words: torch.Tensor) -> torch.Tensor:
    """Bitwise OR of an int32 vector (status words, bits 0..15), on the device."""
    bits = (words.view(-1, 1) >> torch.arange(16, device=words.device, dtype=torch.int32)) & 1
    anyb = bits.amax(0)
    return (anyb << torch.arange(16, device=words.device, dtype=torch.int32)).sum().to(torch.int32).view(1)


def init_distributed(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise torch.distributed from torchrun's environment (RANK/WORLD_SIZE/
    MASTER_ADDR/MASTER_PORT/LOCAL_RANK); returns (rank, world, local_rank)."""
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1 and not dist.is_initialized():
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    elif backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local
