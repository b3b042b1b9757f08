"""Multi-GPU sliding window: one process per GPU, (fold, tile, view) work units sharded, one NCCL exchange.

The reference is single-device (reference ``README.md:209``); its only
coupling between tiles is the additive Gaussian-weighted overlap
(reference ``prediction/sliding_window.py:435-436``), a tile's mirrored views
only meet in the view mean (``mirrored_prediction``, 489-527) and folds are
independent (reference ``prediction/inference.py:65-85``).  So:

* work units are (fold, tile, view) triples, fold outermost, tiles in
  ``itertools.product`` order, views in the reference's mirror order; rank r
  takes the contiguous range ``[r*U/N, (r+1)*U/N)`` (at most one unit more
  than any other rank);
* a rank runs its units in batches of up to 8 consecutive units of one fold
  through the network (a batch may hold the last views of one tile and the
  first of the next), and adds each tile's group of views to its float32
  accumulator as ``(sum of the group's flipped-back logits) / views * g``; the
  normaliser is added once per tile, by the rank holding (fold 0, view 0);
* the accumulator's depth is padded to a multiple of the world size, so two
  NCCL reduce-scatters (logits, normaliser) sum the ranks' contributions and
  leave rank r owning a contiguous z-slab, which it normalises and reduces to
  labels locally.  No data-path collective runs during the tile loop and
  nothing is repacked for the exchange.

A tile whose views are split across ranks sums its view groups separately,
so its float32 rounding differs from the single-device order (the check in
``bench.py`` and the 2-GPU test bound the difference).

The nnunet-fp16 accumulation mode (``predict_volume_fp16_sharded``) depends on
the order of its float16 roundings, so it shards whole folds instead: each
rank runs its folds' float16 windows and normalises each to its float16 crop
exactly as one device does; the folds' halves are broadcast and summed in
fold order on every rank (the same half adds), which gives the single-device
result bit for bit.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction.sliding_window import (
    VolumeAccumulator,
    fold_window_fp16,
    fp16_gaussian,
    mirror_masks,
    pad_minimum,
    tile_offsets,
    validate_request,
)

MAX_BATCH = 8  # network batch: the 8 mirrored views of a tile, or 8 units of one fold


def shard_units(n_tiles: int, n_folds: int, rank: int, world: int, n_views: int = 1) -> list[tuple[int, int, int]]:
    """Contiguous share of the ``(fold, tile, view)`` units of one rank (fold outermost, view fastest)."""
    if world < 1 or not 0 <= rank < world:
        raise ContractError(f"invalid rank {rank} of {world}")
    if n_tiles < 1 or n_folds < 1 or n_views < 1:
        raise ContractError("sharding needs at least one tile, fold and view")
    per_fold = n_tiles * n_views
    units = n_folds * per_fold
    lo, hi = rank * units // world, (rank + 1) * units // world
    return [(u // per_fold, (u % per_fold) // n_views, u % n_views) for u in range(lo, hi)]


def unit_batches(units, max_items: int = MAX_BATCH) -> list[tuple[int, list[tuple[int, int]]]]:
    """Consecutive units of one fold in batches of at most ``max_items``: ``[(fold, [(tile, view), ...]), ...]``."""
    batches: list[tuple[int, list[tuple[int, int]]]] = []
    for fold, tile, view in units:
        if not batches or batches[-1][0] != fold or len(batches[-1][1]) == max_items:
            batches.append((fold, []))
        batches[-1][1].append((tile, view))
    return batches


def tile_groups(items: list[tuple[int, int]]) -> list[tuple[int, int, int]]:
    """Runs of one tile inside a batch: ``[(tile, first item, end item), ...]``."""
    groups: list[tuple[int, int, int]] = []
    for index, (tile, _) in enumerate(items):
        if groups and groups[-1][0] == tile:
            groups[-1] = (tile, groups[-1][1], index + 1)
        else:
            groups.append((tile, index, index + 1))
    return groups


def padded_depth(depth: int, world: int) -> int:
    """Accumulator depth rounded up to a multiple of the world size (the exchange splits it evenly)."""
    return -(-depth // world) * world


def slab_bounds(depth: int, rank: int, world: int) -> tuple[int, int]:
    """z-planes [lo, hi) of the ``depth`` real planes owned by ``rank`` after the exchange."""
    per = -(-depth // world)
    return min(depth, rank * per), min(depth, (rank + 1) * per)


def exchange_slabs(acc: torch.Tensor, normalizer: torch.Tensor, depth: int | None = None, group=None):
    """Sum every rank's ``(Zp, Y, X, C)`` accumulator and ``(Zp, Y, X)`` normaliser; keep this rank's z-slab.

    ``Zp`` must be a multiple of the world size (``padded_depth``); planes at or
    beyond ``depth`` (default ``Zp``) are padding.  Two ``reduce_scatter_tensor``
    calls over the z-major tensors themselves (no packing).  Returns
    ``(z_lo, z_hi, acc_slab, normalizer_slab)``: this rank's real planes
    ``[z_lo, z_hi)``, the slab tensors shaped ``(z_hi - z_lo, Y, X, C)`` and
    ``(z_hi - z_lo, Y, X)`` (views of this rank's share).  Works on any backend
    that implements the collective (NCCL on GPUs, gloo on CPU).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    planes, height, width, classes = (int(s) for s in acc.shape)
    depth = planes if depth is None else int(depth)
    if tuple(normalizer.shape) != (planes, height, width):
        raise ContractError(f"normalizer shape {tuple(normalizer.shape)} does not match "
                            f"accumulator {tuple(acc.shape)}")
    if planes % world != 0 or not 0 < depth <= planes or padded_depth(depth, world) > planes:
        raise ContractError(f"accumulator depth {planes} must be a multiple of the world size {world} "
                            f"covering {depth} real planes")
    if not acc.is_contiguous() or not normalizer.is_contiguous():
        raise ContractError("the exchange needs contiguous accumulators")
    per = planes // world
    acc_mine = torch.empty((per, height, width, classes), dtype=acc.dtype, device=acc.device)
    norm_mine = torch.empty((per, height, width), dtype=normalizer.dtype, device=normalizer.device)
    dist.reduce_scatter_tensor(acc_mine, acc, group=group)
    dist.reduce_scatter_tensor(norm_mine, normalizer, group=group)
    z_lo = min(depth, rank * per)
    z_hi = min(depth, (rank + 1) * per)
    return z_lo, z_hi, acc_mine[: z_hi - z_lo], norm_mine[: z_hi - z_lo]


def run_units(models, volume: torch.Tensor, accumulator: VolumeAccumulator, offsets, units, patch, masks,
              pad_lo=(0, 0, 0), nonfinite: torch.Tensor | None = None) -> None:
    """Run a rank's units: batches of consecutive units of one fold, each tile's view group accumulated."""
    batch = None
    views = len(masks)
    for fold, items in unit_batches(units):
        batch = kernels.gather_tiles(volume, pad_lo, [(offsets[t], masks[v]) for t, v in items], patch, out=batch,
                                     nonfinite=nonfinite)
        model = models[fold]
        features = model.forward_features(batch)
        for tile, lo, hi in tile_groups(items):
            group_views = [v for _, v in items[lo:hi]]
            kernels.accumulate_tile(kernels.lazy_items(features, lo, hi), [masks[v] for v in group_views],
                                    model.seg_weight, model.seg_bias, accumulator.gaussian, accumulator.acc,
                                    accumulator.normalizer, offsets[tile],
                                    add_normalizer=(fold == 0 and 0 in group_views), slope=model.spec.leaky_slope,
                                    view_divisor=views)
        del features


def _any_rank(flags, device, world: int, group):
    """Element-wise logical OR of per-rank flags (one small all-reduce; every rank calls it).

    ``flags``: a bool or a sequence of bools; returns the same shape.
    """
    single = isinstance(flags, bool)
    values = [flags] if single else list(flags)
    if world > 1:
        t = torch.tensor([1 if f else 0 for f in values], dtype=torch.int32, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        values = [bool(v) for v in t.tolist()]
    return values[0] if single else values


def predict_volume_sharded(models, volume: torch.Tensor, *, patch_size, num_classes: int, mirroring_axes=(),
                           step_fraction: float = 0.5, group=None, want_logits: bool = True,
                           label_dtype=torch.uint8):
    """Sharded prediction of a device volume ``(C, *spatial)`` present on every rank.

    Returns ``(z_lo, z_hi, logits_slab, labels_slab, invalid_count)`` for this
    rank's slab of the cropped output (``logits_slab`` is ``(C, z_hi - z_lo, Y, X)``;
    all three tensors are ``None`` when the slab is empty).  Non-finite input
    raises ``ContractError`` on every rank.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    patch, axes = validate_request(tuple(volume.shape), None, patch_size, num_classes, mirroring_axes)
    if volume.dtype != torch.float32 or not volume.is_cuda:
        raise ContractError("expected a float32 CUDA (C, *spatial) volume")
    volume = volume.contiguous()
    pads, crop = pad_minimum(tuple(volume.shape[1:]), patch)
    pad_lo = tuple(a for a, _ in pads)
    spatial = tuple(int(s) + a + b for s, (a, b) in zip(volume.shape[1:], pads))
    offsets = tile_offsets(spatial, patch, step_fraction)
    masks = mirror_masks(axes)
    depth = padded_depth(spatial[0], world)
    units = shard_units(len(offsets), len(models), rank, world, len(masks))
    guarded = any(getattr(m, "range_guarded", False) for m in models)
    nonfinite = torch.zeros((1,), dtype=torch.int32, device=volume.device)
    if guarded:
        kernels.operand_range_events(reset=True)
    accumulator = VolumeAccumulator((depth, *spatial[1:]), num_classes, patch, volume.device)
    run_units(models, volume, accumulator, offsets, units, patch, masks, pad_lo, nonfinite)
    out_of_range = guarded and kernels.operand_range_events(reset=True) > 0
    bad_input, out_of_range = _any_rank([int(nonfinite.item()) != 0, out_of_range], volume.device, world, group)
    if bad_input:
        raise ContractError("expected finite float32 (C, *spatial) input")
    if out_of_range:
        # an activation left the fp16-pair range on some rank: every rank recomputes in split TF32
        accumulator = VolumeAccumulator((depth, *spatial[1:]), num_classes, patch, volume.device)
        run_units([m.range_fallback() for m in models], volume, accumulator, offsets, units, patch, masks, pad_lo)

    if world > 1:
        z_lo, z_hi, acc, normalizer = exchange_slabs(accumulator.acc, accumulator.normalizer, spatial[0], group)
        del accumulator
    else:
        z_lo, z_hi = 0, spatial[0]
        acc, normalizer = accumulator.acc, accumulator.normalizer
    # intersect the slab with the crop window
    c0, c1 = crop[0].start, crop[0].stop
    lo, hi = max(z_lo, c0), min(z_hi, c1)
    if hi <= lo:
        return lo - c0, lo - c0, None, None, None
    crop_lo = (lo - z_lo, crop[1].start, crop[2].start)
    crop_dims = (hi - lo, crop[1].stop - crop[1].start, crop[2].stop - crop[2].start)
    logits, labels, invalid = kernels.normalize_labels(acc, normalizer, crop_lo, crop_dims,
                                                       fold_divisor=float(len(models)), want_logits=want_logits,
                                                       label_dtype=label_dtype)
    return lo - c0, hi - c0, logits, labels, invalid


# ---------------------------------------------------------------------------- nnunet-fp16 across GPUs
def shard_folds(n_folds: int, rank: int, world: int) -> range:
    """Contiguous folds of one rank (``[r*F/N, (r+1)*F/N)``; a rank may get none)."""
    if world < 1 or not 0 <= rank < world or n_folds < 1:
        raise ContractError(f"invalid fold sharding: {n_folds} folds, rank {rank} of {world}")
    return range(rank * n_folds // world, (rank + 1) * n_folds // world)


def fold_owner(fold: int, n_folds: int, world: int) -> int:
    """The rank whose ``shard_folds`` holds ``fold``."""
    for rank in range(world):
        if fold in shard_folds(n_folds, rank, world):
            return rank
    raise ContractError(f"fold {fold} is outside 0..{n_folds - 1}")


def ordered_fold_sum(n_folds: int, mine: dict, fetch, add):
    """Sum fold parts in fold order: ``total = part_0``, then ``add(total, part_f)`` for f = 1..F-1.

    ``mine``: this rank's parts by fold; ``fetch(fold, part_or_None)`` returns
    the fold's part on every rank (a broadcast from its owner); ``add`` adds a
    part into the total in place.
    """
    total = None
    for fold in range(n_folds):
        part = fetch(fold, mine.get(fold))
        if total is None:
            total = part
        else:
            add(total, part)
    return total


def predict_volume_fp16_sharded(models, volume: torch.Tensor, *, patch_size, num_classes: int, mirroring_axes=(),
                                step_fraction: float = 0.5, group=None, want_logits: bool = True,
                                label_dtype=torch.uint8, half_logits: bool = False):
    """nnunet-fp16 fold ensemble of a device volume ``(C, *spatial)`` present on every rank, folds sharded.

    Bit for bit the single-device ``predict_volume(..., accumulation="nnunet-fp16")`` result.  Returns
    ``(logits, labels)`` on rank 0 (logits as float32 values of the halves, or the float16 total with
    ``half_logits``) and ``(None, None)`` on the other ranks.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    patch, axes = validate_request(tuple(volume.shape), None, patch_size, num_classes, mirroring_axes)
    if volume.dtype != torch.float32 or not volume.is_cuda:
        raise ContractError("expected a float32 CUDA (C, *spatial) volume")
    if not models:
        raise ContractError("fold inference requires at least one model")
    volume = volume.contiguous()
    device = volume.device
    pads, crop = pad_minimum(tuple(volume.shape[1:]), patch)
    pad_lo = tuple(a for a, _ in pads)
    spatial = tuple(int(s) + a + b for s, (a, b) in zip(volume.shape[1:], pads))
    lo = [c.start for c in crop]
    dims = [c.stop - c.start for c in crop]
    offsets = tile_offsets(spatial, patch, step_fraction)
    masks = mirror_masks(axes)
    n_folds = len(models)
    mine_folds = shard_folds(n_folds, rank, world)
    gaussian = fp16_gaussian(patch, device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=device)
    nonfinite = torch.zeros((1,), dtype=torch.int32, device=device)

    def run(ms):
        parts = {}
        if len(mine_folds):
            acc = torch.empty((*spatial, num_classes), dtype=torch.float16, device=device)
            normalizer = torch.empty(spatial, dtype=torch.float16, device=device)
            batch = None
            for fold in mine_folds:
                batch = fold_window_fp16(ms[fold], volume, offsets, patch, masks, gaussian, acc, normalizer, pad_lo,
                                         nonfinite, batch)
                part = torch.empty((num_classes, *dims), dtype=torch.float16, device=device)
                kernels.fold_add_fp16(acc, normalizer, lo, dims, part, True, invalid)
                parts[fold] = part
        return parts

    guarded = any(getattr(m, "range_guarded", False) for m in models)
    if guarded:
        kernels.operand_range_events(reset=True)
    parts = run(models)
    out_of_range = guarded and kernels.operand_range_events(reset=True) > 0
    bad_input, out_of_range = _any_rank([int(nonfinite.item()) != 0, out_of_range], device, world, group)
    if bad_input:
        raise ContractError("expected finite float32 (C, *spatial) input")
    if out_of_range:
        parts = run([m.range_fallback() for m in models])

    def fetch(fold, part):
        if world == 1:
            return part
        owner = fold_owner(fold, n_folds, world)
        buf = part if owner == rank else torch.empty((num_classes, *dims), dtype=torch.float16, device=device)
        src = owner if group is None else dist.get_global_rank(group, owner)
        dist.broadcast(buf, src=src, group=group)
        return buf

    total = ordered_fold_sum(n_folds, parts, fetch, lambda t, p: kernels.fold_sum_fp16(t, p, invalid))
    if _any_rank(int(invalid.item()) != 0, device, world, group):
        raise ContractError("sliding-window inference produced non-finite logits")
    if rank != 0:
        return None, None
    logits, labels, bad = kernels.fold_finalize_fp16(total, n_folds, want_logits=want_logits and not half_logits,
                                                     label_dtype=label_dtype)
    if int(bad.item()) != 0:
        raise ContractError("fold averaging produced non-finite logits")
    if half_logits and want_logits:
        logits = total
    return logits, labels
