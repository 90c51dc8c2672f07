"""Data-parallel plumbing for the denoiser: one process per GPU, one independent request per rank.

Independent seeds (or prompts) are the path's natural shards: ranks never exchange activations, so the
data path has no collective. The process group (NCCL on GPUs, gloo on CPU) is used only to agree on
a start point and to take the slowest rank's time, since whole-job throughput is bounded by it.
"""
import os


def world_from_env():
    """(rank, local_rank, world_size) from the torchrun environment (single process: 0, 0, 1)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def shard_requests(global_batch, rank, world):
    """Indices of the requests (seeds) this rank owns: contiguous blocks, sizes differing by at most 1."""
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError("invalid data-parallel layout")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def request_seed(base_seed, request_index):
    """Seed of one request: independent of the world size, so results do not depend on the sharding."""
    return base_seed + request_index


def barrier(group):
    if group is not None:
        group.barrier()


def max_over_ranks(group, value, device=None):
    """Largest value over all ranks (the job's wall time is its slowest rank's)."""
    if group is None:
        return value
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    group.all_reduce(t, op=group.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(group, value, device=None):
    if group is None:
        return value
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    group.all_reduce(t, op=group.ReduceOp.SUM)
    return float(t.item())
