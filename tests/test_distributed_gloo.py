"""Host side of the multi-GPU path on CPU: unit sharding, slab bounds and the
slab exchange collective run as world-size 2 and 3 gloo process groups."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nnunet_mlx_b200.distributed import (
    exchange_slabs,
    padded_depth,
    shard_units,
    slab_bounds,
    tile_groups,
    unit_batches,
)


@pytest.mark.parametrize("tiles,folds,views,world", [(121, 1, 8, 8), (18, 5, 8, 8), (144, 5, 8, 3), (3, 1, 8, 8),
                                                     (7, 2, 4, 2), (5, 3, 1, 4)])
def test_shard_units_cover_every_unit_once_in_order(tiles, folds, views, world):
    shards = [shard_units(tiles, folds, r, world, views) for r in range(world)]
    flat = [u for shard in shards for u in shard]
    assert flat == [(f, t, v) for f in range(folds) for t in range(tiles) for v in range(views)]
    sizes = [len(s) for s in shards]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("tiles,views,world", [(121, 8, 8), (121, 8, 2), (18, 8, 3), (9, 4, 4)])
def test_unit_batches_fill_the_network_batch(tiles, views, world):
    """Every rank runs ceil(units / 8) forwards per fold run; each tile's views are accumulated exactly once."""
    seen = {}
    for rank in range(world):
        units = shard_units(tiles, 1, rank, world, views)
        batches = unit_batches(units)
        assert len(batches) == -(-len(units) // 8)
        assert all(1 <= len(items) <= 8 for _, items in batches)
        for _, items in batches:
            groups = tile_groups(items)
            assert [i for t, lo, hi in groups for i in range(lo, hi)] == list(range(len(items)))
            for tile, lo, hi in groups:
                assert all(items[i][0] == tile for i in range(lo, hi))
                for _, v in items[lo:hi]:
                    seen.setdefault(tile, []).append(v)
    assert seen == {t: list(range(views)) for t in range(tiles)}


def test_unit_batches_never_mix_folds():
    units = shard_units(3, 2, 0, 1, 3)
    for fold, items in unit_batches(units):
        assert all((fold, t, v) in units for t, v in items)
    assert [f for f, _ in unit_batches(units)] == [0, 0, 1, 1]


@pytest.mark.parametrize("depth,world", [(128, 8), (101, 8), (5, 2), (1, 2), (284, 3)])
def test_slab_bounds_partition_the_depth(depth, world):
    bounds = [slab_bounds(depth, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == depth
    for (lo0, hi0), (lo1, hi1) in zip(bounds, bounds[1:]):
        assert lo0 <= hi0 == lo1 <= hi1


def _rank_accumulator(rank: int, shape, classes: int):
    rng = np.random.default_rng(100 + rank)
    acc = torch.from_numpy(rng.standard_normal((*shape, classes)).astype(np.float32))
    norm = torch.from_numpy(rng.uniform(0.1, 1.0, shape).astype(np.float32))
    return acc, norm


def _exchange_worker(rank: int, world: int, port: int, shape, classes: int) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        acc, norm = _rank_accumulator(rank, shape, classes)
        # the accumulator's depth is padded to a multiple of the world size; padding planes hold junk here
        depth = padded_depth(shape[0], world)
        acc_p = torch.full((depth, *shape[1:], classes), 7.0)
        norm_p = torch.full((depth, *shape[1:]), 7.0)
        acc_p[: shape[0]] = acc
        norm_p[: shape[0]] = norm
        z_lo, z_hi, acc_slab, norm_slab = exchange_slabs(acc_p, norm_p, shape[0])
        assert (z_lo, z_hi) == slab_bounds(shape[0], rank, world)
        total_acc = sum(_rank_accumulator(r, shape, classes)[0] for r in range(world))
        total_norm = sum(_rank_accumulator(r, shape, classes)[1] for r in range(world))
        assert acc_slab.shape == (z_hi - z_lo, shape[1], shape[2], classes)
        assert norm_slab.shape == (z_hi - z_lo, shape[1], shape[2])
        torch.testing.assert_close(acc_slab, total_acc[z_lo:z_hi], rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(norm_slab, total_norm[z_lo:z_hi], rtol=1e-6, atol=1e-6)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,shape,classes", [(2, (5, 6, 7), 3), (2, (1, 4, 4), 2), (3, (8, 3, 5), 5)])
def test_exchange_slabs_sums_ranks_and_keeps_the_own_slab(world, shape, classes):
    mp.spawn(_exchange_worker, args=(world, _free_port(), shape, classes), nprocs=world, join=True)


def _any_rank_worker(rank: int, world: int, port: int, flagged: tuple) -> None:
    from nnunet_mlx_b200.distributed import _any_rank

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        assert _any_rank(rank in flagged, torch.device("cpu"), world, None) == bool(flagged)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,flagged", [(2, ()), (2, (1,)), (3, (0, 2))])
def test_range_flag_is_or_reduced_over_ranks(world, flagged):
    """Every rank recomputes in split TF32 when any rank met an out-of-range operand."""
    mp.spawn(_any_rank_worker, args=(world, _free_port(), flagged), nprocs=world, join=True)


@pytest.mark.parametrize("folds,world", [(5, 8), (5, 2), (5, 3), (1, 2), (3, 3)])
def test_shard_folds_partition_in_order(folds, world):
    from nnunet_mlx_b200.distributed import fold_owner, shard_folds

    shards = [list(shard_folds(folds, r, world)) for r in range(world)]
    assert [f for s in shards for f in s] == list(range(folds))
    assert all(fold_owner(f, folds, world) == r for r, s in enumerate(shards) for f in s)


def _fold_sum_worker(rank: int, world: int, port: int, folds: int) -> None:
    from nnunet_mlx_b200.distributed import fold_owner, ordered_fold_sum, shard_folds

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        def part(fold):
            rng = np.random.default_rng(40 + fold)
            return torch.from_numpy(rng.normal(scale=30.0, size=(2, 5, 7)).astype(np.float16))

        def half_add(total, p):
            total.copy_((total.float() + p.float()).half())

        def fetch(fold, mine):
            buf = mine if mine is not None else torch.empty((2, 5, 7), dtype=torch.float16)
            dist.broadcast(buf, src=fold_owner(fold, folds, world))
            return buf

        mine = {f: part(f) for f in shard_folds(folds, rank, world)}
        got = ordered_fold_sum(folds, mine, fetch, half_add)
        expect = part(0).clone()
        for f in range(1, folds):
            half_add(expect, part(f))
        assert torch.equal(got, expect)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,folds", [(2, 5), (3, 5), (2, 1)])
def test_fold_parts_are_summed_in_fold_order_across_ranks(world, folds):
    """The fold-sharded nnunet-fp16 sum equals the single-device half sum bit for bit (CPU half adds here)."""
    mp.spawn(_fold_sum_worker, args=(world, _free_port(), folds), nprocs=world, join=True)
