"""Batch x head sharding of the attention path across ranks (one process per GPU).

Attention (batch, head) units are independent: each rank runs the kernels on
its own units and keeps its dQ/dK/dV, so the data path has no collective. The
only cross-rank traffic is the timing reduction (max over ranks).

    shard_batches(B, world, rank) -> (b0, b1)   contiguous, balanced batch range
    rank_seed(base, rank)                       per-rank input seed (weak scaling)
    max_over_ranks(x)                           max of a float over all ranks
"""
import os


def dist_env():
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_batches(B, world, rank):
    """Contiguous batch range [b0, b1) of `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(B, world)
    b0 = rank * base + min(rank, extra)
    return b0, b0 + base + (1 if rank < extra else 0)


def rank_seed(base, rank):
    return base + 1000003 * rank


def max_over_ranks(x, device=None):
    """Max of a Python float over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
