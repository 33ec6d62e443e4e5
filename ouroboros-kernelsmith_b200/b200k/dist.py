"""Row sharding across the GPUs of one node (one process per GPU).

Every op of the suite is row-independent, so a batch of M rows is split into
contiguous shards and each rank runs the kernels on its own rows with no
data exchange.  The only collective is the reduced cross-entropy: each rank
reduces its shard to [sum of valid-row losses, number of valid rows] (two
fp64 values) and one SUM all-reduce over NCCL (NVLink / NVSwitch) combines
them before the division.
"""
from __future__ import annotations

import torch


def shard_rows(M: int, rank: int, world: int) -> tuple[int, int]:
    """[r0, r1) of rank `rank`: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"b200k: bad rank {rank} of {world}")
    base, extra = divmod(M, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def allreduce_sumcount(sumcount: torch.Tensor, group=None) -> torch.Tensor:
    """In-place SUM all-reduce of a [loss_sum, valid_count] pair over the
    process group (no-op without an initialised group of size > 1)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(sumcount, op=dist.ReduceOp.SUM, group=group)
    return sumcount


def mean_from_sumcount(sumcount: torch.Tensor) -> float:
    """Host-side form of b2k_ce_mean (for CPU tests of the protocol)."""
    s, c = float(sumcount[0]), float(sumcount[1])
    return s / c if c else float("nan")
