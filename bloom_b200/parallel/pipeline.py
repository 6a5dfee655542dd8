"""Pipeline parallelism across GPUs of one box: contiguous layer ranges per
stage, the residual stream handed from stage to stage, sampling on the last
stage and the sampled tokens broadcast back.

The reference's pipeline split is `LayerPlacementStrategy`, a per-layer
CPU / GPU placement run sequentially in one process with tensors copied
between devices (crates/engine/src/core/memory.rs:484-533); its
`ParallelConfig` carries `pp_size` as an enum value only
(crates/engine/src/core/parallelism.rs:21-22).  Here every stage is its own
process on its own GPU with its own scheduler (identical inputs keep the
schedulers in lockstep, as under tensor parallelism), the KV cache of a
stage holds only its layers, and the activations cross NVLink with NCCL
point-to-point sends.  One engine step runs the stages back to back (no
micro-batch interleaving): pipeline parallelism here spreads weights and KV
cache over GPUs for models that do not fit one, it does not add throughput.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch


def layer_range(num_layers: int, stage: int, stages: int) -> Tuple[int, int]:
    """[l0, l1) of one stage: contiguous, sizes differing by at most one
    (earlier stages take the extra layers)."""
    if not 0 <= stage < stages or stages > num_layers:
        raise ValueError(f"stage {stage} of {stages} for {num_layers} layers")
    base, extra = divmod(num_layers, stages)
    l0 = stage * base + min(stage, extra)
    return l0, l0 + base + (1 if stage < extra else 0)


@dataclass
class PPInfo:
    stage: int = 0
    stages: int = 1
    group: object = None       # torch.distributed process group of the pipeline
    ranks: List[int] = field(default_factory=list)  # global rank of every stage

    @property
    def first(self) -> bool:
        return self.stage == 0

    @property
    def last(self) -> bool:
        return self.stage == self.stages - 1

    def send_next(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.send(t.contiguous(), dst=self.ranks[self.stage + 1], group=self.group)

    def recv_prev(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.recv(t, src=self.ranks[self.stage - 1], group=self.group)
        return t

    def broadcast_from_last(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.broadcast(t, src=self.ranks[-1], group=self.group)
        return t

    def max_status(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t


def pipeline_from_world(group=None) -> Optional[PPInfo]:
    """One stage per rank of the (default) process group."""
    import torch.distributed as dist

    if not dist.is_initialized():
        return None
    world = dist.get_world_size(group)
    return PPInfo(stage=dist.get_rank(group), stages=world, group=group, ranks=list(range(world)))
