"""Sharded absmax over several GPUs: one process per GPU, each reducing its own
shard with the side-aware kernel, then one single-float max all-reduce.

The reference has no multi-GPU path (QuickRunCUDA.cpp:286 fixes device 0);
this is the north star's sharded variant.  The exchange is one float per rank,
so NCCL over NVLink/NVSwitch carries it; max over non-negative, non-NaN floats
is exact and order-independent, so the result is bit-identical to a
single-device reduction of the whole stream.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardLayout:
    world: int
    n_per_rank: int
    seed: int
    outlier_rank: int
    outlier_local_index: int
    outlier_sign: int

    def offset(self, rank: int) -> int:
        """First global element index of `rank`'s shard."""
        return rank * self.n_per_rank

    def holds_outlier(self, rank: int) -> bool:
        return rank == self.outlier_rank


def shard_layout(world: int, n_per_rank: int, seed: int, outlier_index_fn) -> ShardLayout:
    """Rank r holds global elements [r*n, (r+1)*n) of the seed's stream; the one
    global outlier sits at outlier_index(seed, world*n), on the rank that holds
    that element.  `outlier_index_fn(seed, total) -> (index, sign)`."""
    if world < 1 or n_per_rank < 1:
        raise ValueError("world and n_per_rank must be positive")
    gi, sign = outlier_index_fn(seed, world * n_per_rank)
    return ShardLayout(world, n_per_rank, seed, gi // n_per_rank, gi % n_per_rank, sign)


def combine_max(value_tensor, group=None) -> None:
    """In-place max all-reduce of a 1-element float tensor (NCCL on GPUs, gloo
    on CPU ranks)."""
    import torch.distributed as dist
    dist.all_reduce(value_tensor, op=dist.ReduceOp.MAX, group=group)


def sharded_absmax(ctx, shard, out, group=None):
    """Side-aware absmax of this rank's shard into `out` (1-element CUDA
    float32 tensor), then the max over all ranks.  Every rank must call it in
    the same order."""
    ctx.absmax(shard, out=out)
    combine_max(out, group)
    return out
