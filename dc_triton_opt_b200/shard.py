"""Multi-GPU plumbing of the DC-attention forward: batch sharding and
max-over-ranks timing.

The op has no cross-batch dependency (an output row [b, t, h] reads only
batch b), so N GPUs split the batch into contiguous slices and run with no
collective on the data path.  ``torch.distributed`` is used only for the
barrier and for reducing per-rank timings.
"""

from __future__ import annotations

import torch


def shard_batch(B: int, world: int, rank: int):
    """Contiguous batch slice [b0, b1) of `rank` out of `world` (even split, the
    remainder going to the first ranks).  Every batch index is owned by exactly
    one rank; ranks past the batch get an empty slice."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(B, world)
    b0 = rank * base + min(rank, rem)
    return b0, b0 + base + (1 if rank < rem else 0)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (e.g. a device-timed duration) over all ranks of
    the default process group; the value itself when not distributed."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], device=device if device is not None else "cpu", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())
