"""Slot sharding across GPUs: one process per GPU, each holding a full weight replica
and a contiguous range of decode slots (slots are independent segments, as the
reference's batching argument rests on, src/decoder.rs:2783-2788).  No collective runs
on the hot path; the only cross-rank operations are the timing barrier and a MAX
reduction of the measured times, both outside the timed region.
"""
from __future__ import annotations


def slot_range(rank: int, world: int, slots_per_rank: int) -> range:
    """Global slot ids owned by `rank` (contiguous, disjoint, covering all ranks)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return range(rank * slots_per_rank, (rank + 1) * slots_per_rank)


def prefix_stream(global_slot: int, refill: int) -> int:
    """Generator stream id of a slot's `refill`-th prefix (independent of the world size,
    so a slot draws the same prefixes whatever GPU it runs on)."""
    return global_slot * 65536 + refill


def max_over_ranks(values, dist=None, device=None):
    """Element-wise MAX of a list of floats over all ranks (identity when not distributed)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return list(values)
    import torch
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
