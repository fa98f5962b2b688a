"""Data parallelism for the training step: the working version of the reference's DataParallel
(om.engine.distributed.ixx:49-188), whose gradient all-reduce is a no-op (:132-161).

One process per GPU. Each rank takes its slice of the global batch (the reference's slicing,
distributed.ixx:80-110: chunk = B // world, the first B % world ranks take one more), runs the
forward/backward on its own GPU, and the gradients are summed across ranks with one NCCL
all-reduce over the flat gradient buffer, then scaled by 1/world before the SGD step, so every
rank applies the mean gradient. BatchNorm statistics stay per rank (the reference's
bSyncBatchNorm flag, distributed.ixx:35, is not implemented there either).

torch.distributed is the plumbing: it owns the process group and the NCCL communicator; the
all-reduce is ordered after this library's backward kernels by running it on the library's
compute stream.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple


@dataclass
class DistributedConfig:
    """distributed.ixx:26-30"""
    nWorldSize: int = 1
    nLocalRank: int = 0
    bSyncBatchNorm: bool = False


def local_slice(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of this rank's samples (distributed.ixx:80-110)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    chunk, rem = divmod(batch, world)
    start = sum(chunk + (1 if r < rem else 0) for r in range(rank))
    return start, start + chunk + (1 if rank < rem else 0)


class DataParallel:
    """Wraps a per-rank training net (plan.Fp32Net) and a process group."""

    def __init__(self, net, config: DistributedConfig, group=None):
        if config.nWorldSize < 1 or not 0 <= config.nLocalRank < config.nWorldSize:
            raise ValueError("DataParallel: bad world size or rank")
        self.net = net
        self.config = config
        self.group = group

    def synchronize_gradients(self, grad_tensor) -> None:
        """Sum the flat gradient across ranks (in place). `grad_tensor` is a torch tensor that
        aliases the net's flat gradient buffer; the caller runs this under the library's
        compute stream so NCCL waits for the backward kernels."""
        if self.config.nWorldSize <= 1:
            return
        import torch.distributed as dist
        dist.all_reduce(grad_tensor, op=dist.ReduceOp.SUM, group=self.group)

    def step(self, lr: float = 0.01, momentum: float = 0.9) -> None:
        self.net.step(lr, momentum, grad_scale=1.0 / self.config.nWorldSize)

    def is_master_rank(self) -> bool:
        return self.config.nLocalRank == 0
