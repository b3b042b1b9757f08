"""Multi-GPU sliding window: one process per GPU, tiles x folds sharded, one NCCL exchange.

The reference is single-device (reference ``README.md:209``); its only
coupling between tiles is the additive Gaussian-weighted overlap
(reference ``prediction/sliding_window.py:435-436``) and folds are
independent (reference ``prediction/inference.py:65-85``).  So:

* work units are (tile, fold) pairs in ``itertools.product`` tile order, fold
  minor; rank r takes the contiguous range ``[r*U/N, (r+1)*U/N)``;
* each rank accumulates its units into its own device float32 accumulator of
  the padded volume (the normaliser is added once per tile, by the tile's
  fold-0 unit);
* one NCCL reduce-scatter over the z-major accumulator sums the ranks'
  contributions and leaves rank r owning a contiguous z-slab, which it
  normalises and reduces to labels locally.  No data-path collective runs
  during the tile loop.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction.sliding_window import (
    VolumeAccumulator,
    mirror_masks,
    pad_minimum,
    tile_offsets,
    validate_request,
)


def shard_units(n_tiles: int, n_folds: int, rank: int, world: int) -> list[tuple[int, int]]:
    """Contiguous share of the (tile, fold) units of one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ContractError(f"invalid rank {rank} of {world}")
    units = n_tiles * n_folds
    lo, hi = rank * units // world, (rank + 1) * units // world
    return [(u // n_folds, u % n_folds) for u in range(lo, hi)]


def slab_bounds(depth: int, rank: int, world: int) -> tuple[int, int]:
    """z-planes [lo, hi) owned by ``rank`` after the reduce-scatter (equal split, padded depth)."""
    per = -(-depth // world)
    return min(depth, rank * per), min(depth, (rank + 1) * per)


def exchange_slabs(acc: torch.Tensor, normalizer: torch.Tensor, group=None):
    """Sum every rank's ``(Z, Y, X, C)`` accumulator and ``(Z, Y, X)`` normaliser; keep this rank's z-slab.

    One ``reduce_scatter_tensor`` over the z-major ``(Z*Y*X, C+1)`` packing
    (z padded to a multiple of the world size).  Returns
    ``(z_lo, z_hi, acc_slab, normalizer_slab)`` with the slab tensors shaped
    ``(z_hi - z_lo, Y, X, C)`` and ``(z_hi - z_lo, Y, X)``.  Works on any
    backend that implements the collective (NCCL on GPUs, gloo on CPU).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    depth, height, width, classes = (int(s) for s in acc.shape)
    if tuple(normalizer.shape) != (depth, height, width):
        raise ContractError(f"normalizer shape {tuple(normalizer.shape)} does not match "
                            f"accumulator {tuple(acc.shape)}")
    z_lo, z_hi = slab_bounds(depth, rank, world)
    per = -(-depth // world)
    plane = height * width
    full = torch.zeros((world * per * plane, classes + 1), dtype=torch.float32, device=acc.device)
    full[: depth * plane, :classes] = acc.reshape(-1, classes)
    full[: depth * plane, classes] = normalizer.reshape(-1)
    mine = torch.empty((per * plane, classes + 1), dtype=torch.float32, device=acc.device)
    dist.reduce_scatter_tensor(mine, full, group=group)
    del full
    mine = mine[: (z_hi - z_lo) * plane]
    acc_slab = mine[:, :classes].contiguous().reshape(z_hi - z_lo, height, width, classes)
    norm_slab = mine[:, classes].contiguous().reshape(z_hi - z_lo, height, width)
    return z_lo, z_hi, acc_slab, norm_slab


def run_units(models, volume: torch.Tensor, accumulator: VolumeAccumulator, offsets, units, patch, masks) -> None:
    current_tile = None
    batch = None
    for tile, fold in units:
        if tile != current_tile:
            batch = kernels.gather_views(volume, offsets[tile], patch, masks, out=batch)
            current_tile = tile
        model = models[fold]
        features = model.forward_features(batch)
        kernels.accumulate_tile(features, masks, model.seg_weight, model.seg_bias, accumulator.gaussian,
                                accumulator.acc, accumulator.normalizer, offsets[tile],
                                add_normalizer=(fold == 0), slope=model.spec.leaky_slope)
        del features


def _any_rank(flag: bool, device, world: int, group) -> bool:
    """Logical OR of a per-rank flag (one small all-reduce; every rank calls it)."""
    if world <= 1:
        return flag
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return bool(t.item())


def predict_volume_sharded(models, volume: torch.Tensor, *, patch_size, num_classes: int, mirroring_axes=(),
                           step_fraction: float = 0.5, group=None, want_logits: bool = True,
                           label_dtype=torch.uint8):
    """Sharded prediction of a device volume ``(C, *spatial)`` present on every rank.

    Returns ``(z_lo, z_hi, logits_slab, labels_slab, invalid_count)`` for this
    rank's slab of the cropped output (``logits_slab`` is ``(C, z_hi - z_lo, Y, X)``;
    all three tensors are ``None`` when the slab is empty).
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    patch, axes = validate_request(tuple(volume.shape), None, patch_size, num_classes, mirroring_axes)
    pads, crop = pad_minimum(tuple(volume.shape[1:]), patch)
    if any(p != (0, 0) for p in pads):
        padded = torch.zeros((volume.shape[0], *(s + a + b for s, (a, b) in zip(volume.shape[1:], pads))),
                             dtype=torch.float32, device=volume.device)
        padded[(slice(None), *crop)] = volume
        volume = padded
    spatial = tuple(int(s) for s in volume.shape[1:])
    offsets = tile_offsets(spatial, patch, step_fraction)
    masks = mirror_masks(axes)
    accumulator = VolumeAccumulator(spatial, num_classes, patch, volume.device)
    units = shard_units(len(offsets), len(models), rank, world)
    guarded = any(getattr(m, "range_guarded", False) for m in models)
    if guarded:
        kernels.operand_range_events(reset=True)
    run_units(models, volume, accumulator, offsets, units, patch, masks)
    if guarded and _any_rank(kernels.operand_range_events(reset=True) > 0, volume.device, world, group):
        # an activation left the fp16-pair range on some rank: every rank recomputes in split TF32
        accumulator = VolumeAccumulator(spatial, num_classes, patch, volume.device)
        run_units([m.range_fallback() for m in models], volume, accumulator, offsets, units, patch, masks)

    if world > 1:
        z_lo, z_hi, acc, normalizer = exchange_slabs(accumulator.acc, accumulator.normalizer, group)
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
