"""The N>1 path on CPU: world_size-2 gloo ranks shard the batch with
dc_triton_opt_b200.shard, each rank computes its slice (with the CPU oracle,
standing in for its GPU), and the gathered result equals the unsharded one —
the op has no cross-batch data.  Also checks the max-over-ranks timing."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dc_triton_opt_b200.shard import max_over_ranks, shard_batch


@pytest.mark.parametrize("B,world", [(16, 8), (5, 2), (3, 4), (64, 8), (1, 2)])
def test_shards_cover_batch_exactly_once(B, world):
    seen = []
    for r in range(world):
        b0, b1 = shard_batch(B, world, r)
        assert 0 <= b0 <= b1 <= B
        seen.extend(range(b0, b1))
    assert sorted(seen) == list(range(B))
    sizes = [shard_batch(B, world, r)[1] - shard_batch(B, world, r)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_bad_rank_rejected():
    with pytest.raises(ValueError):
        shard_batch(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import dc_oracle as O
    B, T, H, D, G, R, W = 3, 40, 8, 16, 2, 1, 12
    q, k, v, pre, post = O.make_inputs(B, T, H, D, G, R, seed=21)
    b0, b1 = shard_batch(B, world, rank)

    def sl(t):
        if t is None:
            return None
        return t[b0:b1] if t.ndim >= 3 else t

    part_pre = O.Terms(identity=pre.identity, w=pre.w, qw1=sl(pre.qw1), qw2=sl(pre.qw2), kw1=sl(pre.kw1),
                       kw2=sl(pre.kw2), qdd=sl(pre.qdd), kdd=sl(pre.kdd))
    part_post = O.Terms(identity=post.identity, w=post.w, qw1=sl(post.qw1), qw2=sl(post.qw2),
                        kw1=sl(post.kw1), kw2=sl(post.kw2), qdd=sl(post.qdd), kdd=sl(post.kdd))
    out = O.dc_attn_oracle(q[b0:b1], k[b0:b1], v[b0:b1], part_pre, part_post, 0.25, W, G)
    # gather the variable-size slices as padded blocks
    pad = np.zeros((B, T, H, D))
    pad[: b1 - b0] = out
    blocks = [torch.zeros(B, T, H, D, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(blocks, torch.from_numpy(pad))
    t = max_over_ranks(10.0 * (rank + 1))
    if rank == 0:
        full = np.concatenate([blocks[r].numpy()[: shard_batch(B, world, r)[1] - shard_batch(B, world, r)[0]]
                               for r in range(world)])
        ref = O.dc_attn_oracle(q, k, v, pre, post, 0.25, W, G)
        np.save(os.path.join(out_dir, "err.npy"), np.array([np.abs(full - ref).max(), t]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    err, t = np.load(tmp_path / "err.npy")
    assert err == 0.0
    assert t == 20.0


@pytest.mark.parametrize("B,G,world", [(1, 8, 8), (2, 8, 8), (3, 8, 8), (1, 4, 8), (64, 1, 8), (2, 1, 8),
                                       (2, 4, 3)])
def test_work_shards_cover_pairs_exactly_once(B, G, world):
    from dc_triton_opt_b200.shard import shard_work
    seen = []
    for r in range(world):
        b0, b1, g0, g1 = shard_work(B, G, world, r)
        assert 0 <= b0 <= b1 <= B and 0 <= g0 <= g1 <= G
        seen.extend((b, g) for b in range(b0, b1) for g in range(g0, g1))
    assert sorted(seen) == [(b, g) for b in range(B) for g in range(G)]


def _group_worker(rank, world, port, out_dir):
    """B=1 < world: the ranks split the head groups of the single batch."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import dc_oracle as O
    from dc_triton_opt_b200.shard import shard_inputs, shard_work
    B, T, H, D, G, R, W = 1, 40, 8, 16, 4, 1, 12
    q, k, v, pre, post = O.make_inputs(B, T, H, D, G, R, seed=33, mix_std=0.1)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a))
    from dc_triton_opt_b200 import DCTerms
    dct = lambda tm: DCTerms(identity=tm.identity, w=t(tm.w), qw1=t(tm.qw1), qw2=t(tm.qw2), kw1=t(tm.kw1),
                             kw2=t(tm.kw2), qdd=t(tm.qdd), kdd=t(tm.kdd))
    shard = shard_work(B, G, world, rank)
    sq, sk, sv, spre, spost, sg = shard_inputs(t(q), t(k), t(v), dct(pre), dct(post), G, shard)
    n = lambda a: None if a is None else a.numpy()
    ot = lambda tm: O.Terms(identity=tm.identity, w=n(tm.w), qw1=n(tm.qw1), qw2=n(tm.qw2), kw1=n(tm.kw1),
                            kw2=n(tm.kw2), qdd=n(tm.qdd), kdd=n(tm.kdd))
    out = O.dc_attn_oracle(n(sq), n(sk), n(sv), ot(spre), ot(spost), 0.25, W, sg)
    b0, b1, g0, g1 = shard
    hpg = H // G
    full = np.zeros((B, T, H, D))
    full[b0:b1, :, g0 * hpg:g1 * hpg] = out
    mask = np.zeros((B, T, H, D))
    mask[b0:b1, :, g0 * hpg:g1 * hpg] = 1.0
    acc, cnt = torch.from_numpy(full), torch.from_numpy(mask)
    dist.all_reduce(acc)
    dist.all_reduce(cnt)
    if rank == 0:
        ref = O.dc_attn_oracle(q, k, v, pre, post, 0.25, W, G)
        np.save(os.path.join(out_dir, "gerr.npy"), np.array([np.abs(acc.numpy() - ref).max(),
                                                              np.abs(cnt.numpy() - 1).max()]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_head_groups(tmp_path):
    world = 2
    mp.spawn(_group_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    err, cover = np.load(tmp_path / "gerr.npy")
    assert cover == 0.0
    assert err < 1e-12
