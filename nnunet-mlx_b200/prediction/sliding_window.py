"""Gaussian sliding-window inference with mirror test-time augmentation, on B200.

API names follow reference ``src/nnunet_mlx/prediction/sliding_window.py``:
``compute_steps`` (32-67), ``gaussian_importance`` (70-93), ``predict_logits``
(116-159), ``predict_device_logits`` (219-254), ``predict_labels`` (312-356),
``_pad_minimum`` (542-562).  The arithmetic is the reference's float32 mode:

* tiles in ``itertools.product`` order of the per-axis starts;
* each tile's prediction is the left-to-right float32 sum of the network
  output and the flipped-back outputs of every non-empty subset of the
  mirroring axes (``combinations`` order), divided by the view count
  (reference 489-527);
* ``acc += pred * g`` and ``normalizer += g`` with the analytic float32
  Gaussian (sigma = patch / 8, maximum 1);
* normalised logits ``acc / normalizer`` (then ``/ n_folds``), label = first
  argmax (reference ``kernels/metal_normalized_labels.py``).

``accumulation="nnunet-fp16"`` is the reference's upstream-compatible mode
(reference 96-113, 415-433; what its MedMLX runners and predict CLI use): the
Gaussian is upstream's scaled impulse response rounded to float16, the window
and normaliser are float16 with every update ``half(f32(acc) + pred * g)``,
each fold is normalised to float16 on its own, and folds are summed in float16
in order and divided in float32 (reference ``inference.py:65-90``).  That mode
keeps one float16 window per fold instead of the shared float32 accumulator.

Execution is B200-native: the input volume is uploaded once, every mirrored
view of a tile runs as one batch through the network, the segmentation head
+ flip-back + view mean + Gaussian accumulation is one fused kernel per tile
and fold, and the full-volume float32 accumulator stays resident in HBM (the
reference's slab windowing exists to bound unified memory; additions per
voxel and their order are the same).  Folds share the accumulator:
sum_f(L_f) / normalizer / n_folds equals the reference's per-fold normalised
average up to float32 rounding.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from functools import lru_cache
from itertools import combinations, product

import numpy as np
import torch

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError


def _axis_steps(image: int, patch: int, step_fraction: float) -> tuple[int, ...]:
    if image < patch:
        raise ContractError(f"padded image dimension {image} is smaller than patch {patch}")
    count = int(np.ceil((image - patch) / (patch * step_fraction))) + 1
    maximum = image - patch
    actual = maximum / (count - 1) if count > 1 else 0.0
    return tuple(round(actual * index) for index in range(count))


def compute_steps(image_size: Sequence[int], patch_size: Sequence[int], *,
                  step_fraction: float = 0.5) -> tuple[tuple[int, ...], ...]:
    """Per-axis tile start offsets (upstream ``compute_steps_for_sliding_window``)."""
    if not 0 < step_fraction <= 1:
        raise ContractError(f"step_fraction must be in (0, 1], got {step_fraction}")
    if len(image_size) not in (2, 3) or len(patch_size) != len(image_size):
        raise ContractError("sliding-window inference requires matching 2-D or 3-D shapes")
    return tuple(_axis_steps(int(i), int(p), step_fraction) for i, p in zip(image_size, patch_size))


@lru_cache(maxsize=8)
def gaussian_importance(patch_size: tuple[int, ...]) -> np.ndarray:
    """Float32 separable Gaussian, sigma = size / 8, centre size // 2, max 1, zeros -> tiny."""
    if any(size < 1 for size in patch_size):
        raise ContractError(f"invalid patch size {patch_size}")
    exponent = np.zeros(patch_size, dtype=np.float32)
    for axis, size in enumerate(patch_size):
        coordinates = np.arange(size, dtype=np.float32)
        shape = tuple(size if i == axis else 1 for i in range(len(patch_size)))
        exponent += (((coordinates - size // 2) / (size / 8)) ** 2).reshape(shape)
    values = np.exp(-0.5 * exponent).astype(np.float32, copy=False)
    values /= np.float32(values.max())
    values[values == 0] = np.finfo(np.float32).tiny
    values.setflags(write=False)
    return values


@lru_cache(maxsize=8)
def nnunet_fp16_gaussian(patch_size: tuple[int, ...]) -> np.ndarray:
    """Upstream nnU-Net's importance map: a unit impulse at ``size // 2`` filtered by a Gaussian of
    sigma ``size / 8`` per axis (constant mode), scaled to maximum 10 and cast to float16; entries
    that round to zero take the smallest nonzero value (reference sliding_window.py:96-113)."""
    from scipy.ndimage import gaussian_filter

    patch = tuple(int(v) for v in patch_size)
    if any(size < 1 for size in patch):
        raise ContractError(f"invalid patch size {patch}")
    impulse = np.zeros(patch)
    impulse[tuple(size // 2 for size in patch)] = 1
    weights = gaussian_filter(impulse, [size / 8 for size in patch], mode="constant")
    rounded = (weights / (weights.max() / 10)).astype(np.float16)
    rounded[rounded == 0] = rounded[rounded != 0].min()
    rounded.setflags(write=False)
    return rounded


ACCUMULATIONS = ("float32", "nnunet-fp16")


def mirror_masks(axes: Sequence[int]) -> list[int]:
    """Flip bitmasks of the views, in the reference's view order."""
    masks = [0]
    for count in range(1, len(axes) + 1):
        for selected in combinations(tuple(axes), count):
            masks.append(sum(1 << a for a in selected))
    return masks


def pad_minimum(shape: Sequence[int], patch: Sequence[int]):
    """Zero padding before/after per axis so every axis is >= patch (odd voxel after)."""
    pads, crop = [], []
    for size, minimum in zip(shape, patch):
        total = max(0, minimum - size)
        before = total // 2
        pads.append((before, total - before))
        crop.append(slice(before, before + size))
    return pads, tuple(crop)


def validate_request(data_shape, dtype, patch_size, num_classes, mirroring_axes):
    spatial_dims = len(data_shape) - 1
    if spatial_dims != 3:
        raise ContractError(f"expected float32 (C, *spatial) 3-D input, got {tuple(data_shape)}")
    patch = tuple(int(v) for v in patch_size)
    if len(patch) != 3 or any(v < 1 for v in patch):
        raise ContractError(f"invalid patch size {patch}")
    if num_classes < 1:
        raise ContractError("sliding-window inference requires at least one output channel")
    axes = tuple(int(a) for a in mirroring_axes)
    if any(a not in range(3) for a in axes) or len(set(axes)) != len(axes):
        raise ContractError(f"invalid mirroring axes {axes}")
    return patch, axes


def _to_device_volume(data, device) -> torch.Tensor:
    if isinstance(data, torch.Tensor):
        volume = data
    else:
        array = np.asarray(data)
        if array.dtype != np.float32:
            raise ContractError("expected finite float32 (C, *spatial) input")
        volume = torch.from_numpy(np.ascontiguousarray(array))
    if volume.dtype != torch.float32:
        raise ContractError("expected finite float32 (C, *spatial) input")
    # finiteness is checked by the tile gather as it reads the volume (one count per volume)
    return volume.to(device, non_blocking=True).contiguous()


def tile_offsets(spatial, patch, step_fraction: float) -> list[tuple[int, int, int]]:
    steps = compute_steps(spatial, patch, step_fraction=step_fraction)
    return [tuple(int(v) for v in o) for o in product(*steps)]


class VolumeAccumulator:
    """Device-resident float32 logits accumulator + Gaussian normaliser for one padded volume."""

    def __init__(self, padded_spatial, num_classes: int, patch, device) -> None:
        self.shape = tuple(int(s) for s in padded_spatial)
        self.acc = torch.zeros((*self.shape, num_classes), dtype=torch.float32, device=device)
        self.normalizer = torch.zeros(self.shape, dtype=torch.float32, device=device)
        # the cached map is read-only: hand torch a writable copy of it
        self.gaussian = torch.from_numpy(np.array(gaussian_importance(tuple(patch)), dtype=np.float32)).to(device)


def run_tiles(models, volume: torch.Tensor, acc: VolumeAccumulator, offsets, patch, masks,
              batch_buffer: torch.Tensor | None = None, pad_lo=(0, 0, 0),
              nonfinite: torch.Tensor | None = None) -> None:
    """Run every fold on every tile in ``offsets`` and accumulate (the hot loop).

    ``offsets`` are coordinates of ``volume`` zero-padded by ``pad_lo`` (read
    unpadded by the gather); ``nonfinite`` counts non-finite input values.
    """
    for offset in offsets:
        batch = kernels.gather_tiles(volume, pad_lo, [(offset, m) for m in masks], patch, out=batch_buffer,
                                     nonfinite=nonfinite)
        batch_buffer = batch
        for index, model in enumerate(models):
            features = model.forward_features(batch)
            kernels.accumulate_tile(features, masks, model.seg_weight, model.seg_bias, acc.gaussian, acc.acc,
                                    acc.normalizer, offset, add_normalizer=(index == 0),
                                    slope=model.spec.leaky_slope)
            del features


def range_guarded(models, run, nonfinite: torch.Tensor | None = None):
    """``run(models)``, recomputed with the split-TF32 twins when an fp16-pair operand was out of range.

    Networks in the default ``fp32`` precision compute with fp16 hi/lo operand
    pairs, exact to float32 level while every activation stays below 65504 in
    magnitude; the operand preparation counts the elements that do not.  The
    count is read once per volume (one device synchronisation), after the
    gather's count of non-finite input values (``nonfinite``), which raises.
    """
    guarded = any(getattr(m, "range_guarded", False) for m in models)
    if guarded:
        kernels.operand_range_events(reset=True)
    result = run(models)
    if nonfinite is not None and int(nonfinite.item()) != 0:
        raise ContractError("expected finite float32 (C, *spatial) input")
    if guarded and kernels.operand_range_events(reset=True) > 0:
        result = run([m.range_fallback() for m in models])
    return result


def predict_volume(models, data, *, patch_size, num_classes: int, mirroring_axes=(), step_fraction: float = 0.5,
                   want_logits: bool = True, label_dtype=torch.uint8, device=None, accumulation: str = "float32",
                   half_logits: bool = False):
    """Device logits ``(C, *spatial)`` (float32) and labels for a preprocessed ``(C, *spatial)`` volume.

    With ``accumulation="nnunet-fp16"`` the logits are the float16 fold average
    (as float32 values, or the float16 tensor itself when ``half_logits``).
    """
    if not models:
        raise ContractError("fold inference requires at least one model")
    _check_accumulation(accumulation)
    shape = tuple(data.shape)
    patch, axes = validate_request(shape, None, patch_size, num_classes, mirroring_axes)
    device = torch.device(device) if device is not None else models[0].device
    volume = _to_device_volume(data, device)
    # axes shorter than the patch are zero-padded virtually: the gather reads the unpadded volume
    pads, crop = pad_minimum(shape[1:], patch)
    pad_lo = tuple(a for a, _ in pads)
    spatial = tuple(s + a + b for s, (a, b) in zip(shape[1:], pads))
    masks = mirror_masks(axes)
    lo = [c.start for c in crop]
    dims = [c.stop - c.start for c in crop]
    nonfinite = torch.zeros((1,), dtype=torch.int32, device=device)
    if accumulation == "nnunet-fp16":
        return range_guarded(models, lambda ms: _predict_volume_fp16(
            ms, volume, spatial, num_classes, patch, masks, step_fraction, lo, dims, want_logits, label_dtype,
            half_logits, pad_lo, nonfinite), nonfinite)

    def run(ms):
        accumulator = VolumeAccumulator(spatial, num_classes, patch, device)
        run_tiles(ms, volume, accumulator, tile_offsets(spatial, patch, step_fraction), patch, masks,
                  pad_lo=pad_lo, nonfinite=nonfinite)
        return kernels.normalize_labels(accumulator.acc, accumulator.normalizer, lo, dims,
                                        fold_divisor=float(len(ms)), want_logits=want_logits, label_dtype=label_dtype)

    logits, labels, invalid = range_guarded(models, run, nonfinite)
    if int(invalid.item()) != 0:
        raise ContractError("sliding-window inference produced non-finite logits")
    return logits, labels


def fold_window_fp16(model, volume, offsets, patch, masks, gaussian, acc, normalizer, pad_lo=(0, 0, 0),
                     nonfinite=None, batch=None):
    """One fold's float16 window + normaliser over every tile (nnunet-fp16; ``acc`` / ``normalizer`` are zeroed
    first).  Returns the reusable gather buffer."""
    acc.zero_()
    normalizer.zero_()
    for offset in offsets:
        batch = kernels.gather_tiles(volume, pad_lo, [(offset, m) for m in masks], patch, out=batch,
                                     nonfinite=nonfinite)
        features = model.forward_features(batch)
        kernels.accumulate_tile(features, masks, model.seg_weight, model.seg_bias, gaussian, acc, normalizer, offset,
                                add_normalizer=True, slope=model.spec.leaky_slope)
        del features
    return batch


def fp16_gaussian(patch, device) -> torch.Tensor:
    return torch.from_numpy(nnunet_fp16_gaussian(tuple(patch)).astype(np.float32)).to(device)


def _predict_volume_fp16(models, volume, spatial, num_classes, patch, masks, step_fraction, lo, dims, want_logits,
                         label_dtype, half_logits, pad_lo=(0, 0, 0), nonfinite=None):
    """nnunet-fp16: per fold a float16 window + normaliser, normalised to float16 and summed in fold order."""
    device = volume.device
    gaussian = fp16_gaussian(patch, device)
    offsets = tile_offsets(spatial, patch, step_fraction)
    total = torch.empty((num_classes, *dims), dtype=torch.float16, device=device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=device)
    acc = torch.empty((*spatial, num_classes), dtype=torch.float16, device=device)
    normalizer = torch.empty(spatial, dtype=torch.float16, device=device)
    batch = None
    for index, model in enumerate(models):
        batch = fold_window_fp16(model, volume, offsets, patch, masks, gaussian, acc, normalizer, pad_lo,
                                 nonfinite if index == 0 else None, batch)
        kernels.fold_add_fp16(acc, normalizer, lo, dims, total, index == 0, invalid)
    if nonfinite is not None and int(nonfinite.item()) != 0:
        raise ContractError("expected finite float32 (C, *spatial) input")
    if int(invalid.item()) != 0:
        raise ContractError("sliding-window inference produced non-finite logits")
    logits, labels, invalid = kernels.fold_finalize_fp16(total, len(models), want_logits=want_logits and not half_logits,
                                                         label_dtype=label_dtype)
    if int(invalid.item()) != 0:
        raise ContractError("fold averaging produced non-finite logits")
    if half_logits and want_logits:
        logits = total
    return logits, labels


def predict_logits(model, data_channels_first, *, patch_size, num_classes: int, mirroring_axes=(),
                   step_fraction: float = 0.5, accumulation: str = "float32") -> np.ndarray:
    """Host float32 ``(num_classes, *spatial)`` logits (reference sliding_window.py:116-159).

    ``nnunet-fp16`` logits are the float16-rounded values, returned as float32.
    """
    _check_accumulation(accumulation)
    models = model if isinstance(model, (list, tuple)) else [model]
    logits, _ = predict_volume(models, data_channels_first, patch_size=patch_size, num_classes=num_classes,
                               mirroring_axes=mirroring_axes, step_fraction=step_fraction, label_dtype=None,
                               accumulation=accumulation)
    return kernels.to_host(logits)


def predict_device_logits(model, data_channels_first, *, patch_size, num_classes: int, mirroring_axes=(),
                          step_fraction: float = 0.5, accumulation: str = "float32") -> torch.Tensor:
    """Device logits as channels-last ``(*spatial, C)`` (a view of the channel-first result);
    float16 for ``nnunet-fp16`` (reference 219-254)."""
    _check_accumulation(accumulation)
    models = model if isinstance(model, (list, tuple)) else [model]
    logits, _ = predict_volume(models, data_channels_first, patch_size=patch_size, num_classes=num_classes,
                               mirroring_axes=mirroring_axes, step_fraction=step_fraction, label_dtype=None,
                               accumulation=accumulation, half_logits=True)
    return logits.permute(1, 2, 3, 0)


def predict_labels(model, data_channels_first, *, patch_size, num_classes: int, mirroring_axes=(),
                   step_fraction: float = 0.5, accumulation: str = "float32") -> np.ndarray:
    """Host uint16 labels; only labels cross to the host (reference 312-356)."""
    _check_accumulation(accumulation)
    models = model if isinstance(model, (list, tuple)) else [model]
    _, labels = predict_volume(models, data_channels_first, patch_size=patch_size, num_classes=num_classes,
                               mirroring_axes=mirroring_axes, step_fraction=step_fraction, want_logits=False,
                               label_dtype=torch.uint16 if num_classes > 255 else torch.uint8,
                               accumulation=accumulation)
    return kernels.to_host(labels).astype(np.uint16)


def _check_accumulation(accumulation: str) -> None:
    if accumulation not in ACCUMULATIONS:
        raise ContractError(f"unsupported sliding-window accumulation {accumulation!r}")


def volume_work(shape, patch, step_fraction: float, views: int, folds: int) -> dict:
    """Tile / forward counts of a volume (for reporting)."""
    pads, _ = pad_minimum(shape, patch)
    spatial = [s + a + b for s, (a, b) in zip(shape, pads)]
    tiles = len(tile_offsets(spatial, patch, step_fraction))
    return {"tiles": tiles, "forwards": tiles * views * folds, "voxels": int(math.prod(shape))}
