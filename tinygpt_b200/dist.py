"""Batch partitioning across the GPUs of one box (one process per GPU).

Rows are independent, so the batch is split into contiguous slices, one per
rank, with no collective on the data path; a caller that wants every rank to
hold every id gathers them afterwards (gather_ids).  torch.distributed provides
the process group (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, start+count) of `rank` when `total` rows are split contiguously;
    the first total % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_ids(ids_local, total: int, group=None):
    """All-gather per-rank id slices (contiguous shards of `total` rows) into the
    full [total] vector on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    counts = [shard_rows(total, world, r)[1] for r in range(world)]
    width = max(counts) if counts else 0
    pad = torch.full((width,), -1, dtype=ids_local.dtype, device=ids_local.device)
    pad[: ids_local.numel()] = ids_local
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad, group=group)
    return torch.cat([o[:c] for o, c in zip(out, counts)])


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The maximum of a per-rank float (e.g. a step time) over all ranks."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
