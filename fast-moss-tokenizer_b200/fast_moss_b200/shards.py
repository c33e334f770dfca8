"""Data-parallel sharding of independent clips, streams or frame batches.

The hot path has no exchange step: clips, streams and frame batches are
independent, so one process per GPU takes a contiguous shard and no
collective touches the data.  The only collectives are the ones a driver
uses around a timed region: a barrier and a max over ranks of the elapsed
time.
"""

import torch


def shard_bounds(total, rank, world):
    """[start, end) of `rank`'s contiguous share of `total` items; the first
    `total % world` ranks take one extra item, so shares differ by at most 1."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request: total={total}, rank={rank}, world={world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(tensor, rank, world, dim=0):
    """The rank's contiguous slice of `tensor` along `dim` (a view)."""
    start, end = shard_bounds(tensor.shape[dim], rank, world)
    return tensor.narrow(dim, start, end - start)


def max_over_ranks(values, device=None):
    """Elementwise maximum of a list of floats over all ranks of the default
    process group (returned as floats); the identity without one."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
