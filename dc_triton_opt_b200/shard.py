"""Multi-GPU plumbing of the DC-attention forward: batch and head-group
sharding, and max-over-ranks timing.

The op has no cross-shard dependency: an output row [b, t, h] reads only
batch b and the heads of h's group (composition mixes heads inside a group
only).  N GPUs therefore split the work into contiguous batch slices, and into
contiguous head-group ranges as well when the batch alone has fewer entries
than ranks, and run with no collective on the data path.
``torch.distributed`` is used only for the barrier and for reducing per-rank
timings.
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


def shard_work(B: int, G: int, world: int, rank: int):
    """Shard (b0, b1, g0, g1) of `rank`: batches [b0, b1) x head groups [g0, g1).

    With B >= world the batch alone is split (every rank owns all G groups of
    its slice, as :func:`shard_batch`).  Otherwise the B x G (batch, group)
    pairs are split into `world` contiguous runs in batch-major order, cut so
    that each rank's run stays inside one batch (ranks are assigned to batches
    in proportion, then each batch's groups are split among its ranks).  Every
    (batch, group) pair is owned by exactly one rank; ranks beyond B*G pairs
    get an empty shard (b0 == b1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if B >= world or G == 1:
        b0, b1 = shard_batch(B, world, rank)
        return b0, b1, 0, G
    # fewer batches than ranks: each batch gets world // B (+1) ranks, which split its groups
    b = 0
    r0 = 0
    for bb in range(B):
        nr = world // B + (1 if bb < world % B else 0)
        if rank < r0 + nr:
            b = bb
            break
        r0 += nr
    nr = world // B + (1 if b < world % B else 0)
    g0, g1 = shard_batch(G, nr, rank - r0)
    if g0 == g1:
        return b, b, 0, 0
    return b, b + 1, g0, g1


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (e.g. a device-timed duration) over all ranks of
    the default process group; the value itself when not distributed."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], device=device if device is not None else "cpu", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def shard_inputs(q, k, v, pre, post, G: int, shard):
    """The inputs of one shard (b0, b1, g0, g1) as contiguous tensors: q, k, v
    [b1-b0, T, (g1-g0)*HPG, D], the term sets restricted to those batches and
    heads (static mixes to groups [g0, g1)), and the shard's group count.  Its
    forward equals rows [b0, b1) x heads [g0*HPG, g1*HPG) of the full output."""
    from .api import DCTerms
    b0, b1, g0, g1 = shard
    H = q.shape[2]
    hpg = H // G
    h0, h1 = g0 * hpg, g1 * hpg
    cut = lambda t: t[b0:b1, :, h0:h1].contiguous()

    def terms(tm):
        if tm is None:
            return None
        f = lambda t, sl: None if t is None else sl(t)
        return DCTerms(identity=tm.identity, w=f(tm.w, lambda t: t[g0:g1].contiguous()),
                       qw1=f(tm.qw1, cut), qw2=f(tm.qw2, lambda t: t[b0:b1, :, :, h0:h1].contiguous()),
                       kw1=f(tm.kw1, cut), kw2=f(tm.kw2, lambda t: t[b0:b1, :, :, h0:h1].contiguous()),
                       qdd=f(tm.qdd, cut), kdd=f(tm.kdd, cut), qmat=f(tm.qmat, cut))

    return cut(q), cut(k), cut(v), terms(pre), terms(post), g1 - g0
