"""Multi-GPU plumbing for batch-sharded inference (no data-path collectives).

Samples are independent, so each rank (one process per GPU) takes a
contiguous slice of the batch and runs it with its own arena.  The only
cross-rank traffic is control: barriers and the max-over-ranks reduction of
device times, through ``torch.distributed`` (NCCL on GPUs, gloo on CPU for
tests).
"""

from __future__ import annotations

from typing import Tuple


def shard(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous rows [start, stop) of rank ``rank`` (ceil split, first ranks larger)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def rows_for(scaling: str, batch: int, world: int, rank: int) -> Tuple[int, int, int]:
    """(global rows, start, count): weak scaling keeps ``batch`` per rank,
    strong scaling splits a global ``batch``."""
    if scaling == "weak":
        return batch * world, rank * batch, batch
    s, e = shard(batch, world, rank)
    return batch, s, e - s


def reduce_max(value: float, device: str = "cpu") -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
