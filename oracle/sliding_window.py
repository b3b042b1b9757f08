"""NumPy float32 restatement of the reference sliding-window predictor -- TEST INFRASTRUCTURE.

Follows reference ``src/nnunet_mlx/prediction/sliding_window.py``:

* ``compute_steps`` / ``_axis_steps`` (32-67): ``n = ceil((img - P) / (P * step)) + 1``
  starts, ``round(i * (img - P) / (n - 1))`` with Python's round-half-even;
* ``gaussian_importance`` (70-93): separable ``exp(-1/2 * sum(((i - P//2) / (P/8))^2))``
  in float32, divided by its maximum, exact zeros replaced by float32 ``tiny``;
* ``_pad_minimum`` (542-562): zero padding of axes shorter than the patch, odd
  voxel after;
* ``mirrored_prediction`` (489-527): ``m(x)`` plus ``flip(m(flip(x)))`` for every
  non-empty subset of the mirroring axes in ``combinations`` order, summed
  left to right in float32, divided by the view count;
* ``_accumulate_logits`` (359-460): tiles in ``itertools.product`` order,
  ``logits[win] += pred * g`` and ``normalizer[win] += g`` in float32.  The
  reference's slab windowing performs the same additions in the same order as
  this full-volume accumulator (its docstring, 370-382);
* ``predict_logits`` (116-216): ``logits / normalizer`` in float32, cropped,
  channel-first;
* ``average_fold_logits`` (reference ``prediction/inference.py:25-90``): fold
  sum in order, then ``/ n_folds`` in float32;
* ``normalized_labels`` (reference ``kernels/metal_normalized_labels.py:19-98``):
  first maximum of ``logits / normalizer``; a non-finite or non-positive
  denominator or a non-finite quotient gives 65535.

Only tests, ``smoke()`` and the bench CPU baseline may use this module.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from itertools import combinations, product

import numpy as np

INVALID_LABEL = 65535


def axis_steps(image: int, patch: int, step_fraction: float) -> tuple[int, ...]:
    if image < patch:
        raise ValueError(f"padded image dimension {image} is smaller than patch {patch}")
    count = int(math.ceil((image - patch) / (patch * step_fraction))) + 1
    maximum = image - patch
    actual = maximum / (count - 1) if count > 1 else 0.0
    return tuple(round(actual * index) for index in range(count))


def compute_steps(image_size, patch_size, step_fraction: float = 0.5):
    if not 0 < step_fraction <= 1:
        raise ValueError("step_fraction must be in (0, 1]")
    return tuple(axis_steps(int(i), int(p), step_fraction) for i, p in zip(image_size, patch_size))


def gaussian_importance(patch_size: Sequence[int]) -> np.ndarray:
    patch_size = tuple(int(s) for s in patch_size)
    exponent = np.zeros(patch_size, dtype=np.float32)
    for axis, size in enumerate(patch_size):
        center = size // 2
        sigma = size / 8
        coords = np.arange(size, dtype=np.float32)
        shape = tuple(size if i == axis else 1 for i in range(len(patch_size)))
        exponent += (((coords - center) / sigma) ** 2).reshape(shape)
    values = np.exp(-0.5 * exponent).astype(np.float32, copy=False)
    values /= np.float32(values.max())
    values[values == 0] = np.finfo(np.float32).tiny
    return values


def pad_minimum(data: np.ndarray, patch: Sequence[int]):
    padding = [(0, 0)]
    crop = []
    for size, minimum in zip(data.shape[1:], patch):
        total = max(0, minimum - size)
        before = total // 2
        padding.append((before, total - before))
        crop.append(slice(before, before + size))
    return np.pad(data, padding), tuple(crop)


def mirror_subsets(axes: Sequence[int]) -> list[tuple[int, ...]]:
    """The view order of ``mirrored_prediction``: (), then combinations by size."""
    views: list[tuple[int, ...]] = [()]
    for count in range(1, len(axes) + 1):
        views.extend(combinations(tuple(axes), count))
    return views


def mirrored_prediction(model: Callable[[np.ndarray], np.ndarray], tile: np.ndarray,
                        axes: Sequence[int]) -> np.ndarray:
    """``tile``: channels-last ``(1, *patch, C_in)``; returns ``(1, *patch, C)`` float32."""
    views = mirror_subsets(axes)
    prediction = np.asarray(model(tile), dtype=np.float32)
    for selected in views[1:]:
        flip_axes = tuple(a + 1 for a in selected)
        mirrored = np.ascontiguousarray(np.flip(tile, axis=flip_axes))
        current = np.flip(np.asarray(model(mirrored), dtype=np.float32), axis=flip_axes)
        prediction = prediction + current
    if len(views) == 1:
        return prediction
    return (prediction / np.float32(len(views))).astype(np.float32)


def accumulate(model, padded_cf: np.ndarray, patch, axes, num_classes: int, step_fraction: float):
    """Full-volume float32 accumulation; returns channels-last ``(logits, normalizer)``."""
    spatial = padded_cf.shape[1:]
    steps = compute_steps(spatial, patch, step_fraction)
    g = gaussian_importance(patch)[..., None]
    volume = np.ascontiguousarray(np.moveaxis(padded_cf, 0, -1))
    logits = np.zeros((*spatial, num_classes), dtype=np.float32)
    normalizer = np.zeros((*spatial, 1), dtype=np.float32)
    for offsets in product(*steps):
        sl = tuple(slice(o, o + p) for o, p in zip(offsets, patch))
        pred = mirrored_prediction(model, volume[sl][None], axes)
        logits[sl] += pred[0] * g
        normalizer[sl] += g
    return logits, normalizer


def nnunet_fp16_gaussian(patch_size: Sequence[int]) -> np.ndarray:
    """Upstream's importance map (reference sliding_window.py:96-113): impulse at ``size // 2``,
    scipy ``gaussian_filter`` with sigma ``size / 8`` (constant mode), scaled to max 10, cast to
    float16, zeros replaced by the smallest nonzero value."""
    from scipy.ndimage import gaussian_filter

    patch = tuple(int(p) for p in patch_size)
    impulse = np.zeros(patch)
    impulse[tuple(s // 2 for s in patch)] = 1
    weights = gaussian_filter(impulse, [s / 8 for s in patch], mode="constant")
    rounded = (weights / (weights.max() / 10)).astype(np.float16)
    rounded[rounded == 0] = rounded[rounded != 0].min()
    return rounded


def accumulate_fp16(model, padded_cf: np.ndarray, patch, axes, num_classes: int, step_fraction: float):
    """nnunet-fp16 window (reference sliding_window.py:415-433): float16 logits and normaliser, each
    tile ``half(f32(logits) + pred * g32)`` and ``half(f32(norm) + g32)`` (IEEE half add)."""
    spatial = padded_cf.shape[1:]
    steps = compute_steps(spatial, patch, step_fraction)
    g16 = nnunet_fp16_gaussian(patch)[..., None]
    g32 = g16.astype(np.float32)
    volume = np.ascontiguousarray(np.moveaxis(padded_cf, 0, -1))
    logits = np.zeros((*spatial, num_classes), dtype=np.float16)
    normalizer = np.zeros((*spatial, 1), dtype=np.float16)
    for offsets in product(*steps):
        sl = tuple(slice(o, o + p) for o, p in zip(offsets, patch))
        pred = mirrored_prediction(model, volume[sl][None], axes)
        weighted = (pred[0] * g32).astype(np.float32)
        logits[sl] = (logits[sl].astype(np.float32) + weighted).astype(np.float16)
        normalizer[sl] = (normalizer[sl].astype(np.float32) + g32).astype(np.float16)
    return logits, normalizer


def predict_logits(model, data_cf: np.ndarray, *, patch_size, num_classes: int,
                   mirroring_axes=(), step_fraction: float = 0.5, accumulation: str = "float32") -> np.ndarray:
    """Channel-first ``(C, *spatial)`` normalized logits (reference 116-216): float32, or the
    float16 values ``half(f32(logits) / f32(norm))`` for ``nnunet-fp16`` (as a float16 array)."""
    patch = tuple(int(p) for p in patch_size)
    padded, crop = pad_minimum(np.asarray(data_cf, dtype=np.float32), patch)
    if accumulation == "nnunet-fp16":
        logits, normalizer = accumulate_fp16(model, padded, patch, tuple(mirroring_axes), num_classes,
                                             step_fraction)
        normalized = (logits.astype(np.float32) / normalizer.astype(np.float32)).astype(np.float16)
    else:
        logits, normalizer = accumulate(model, padded, patch, tuple(mirroring_axes), num_classes, step_fraction)
        normalized = (logits / normalizer).astype(np.float32)
    return np.ascontiguousarray(np.moveaxis(normalized[crop], -1, 0))


def average_fold_logits(models, data_cf, *, patch_size, num_outputs, mirroring_axes=(),
                        step_fraction: float = 0.5, accumulation: str = "float32") -> np.ndarray:
    """Fold ensemble (reference inference.py:65-90): float32 sum / n, or for ``nnunet-fp16`` each
    fold rounded to float16, summed in fold order in float16 and divided by float32(n) (float16)."""
    folds = [predict_logits(model, data_cf, patch_size=patch_size, num_classes=num_outputs,
                            mirroring_axes=mirroring_axes, step_fraction=step_fraction,
                            accumulation=accumulation) for model in models]
    return average_folds(folds, accumulation)


def average_folds(folds, accumulation: str = "float32") -> np.ndarray:
    """The fold-sum-and-divide step alone, on given per-fold logits."""
    half = accumulation == "nnunet-fp16"
    total = None
    for current in folds:
        values = np.asarray(current, dtype=np.float16 if half else np.float32)
        if total is None:
            total = values.copy()
        elif half:
            total = (total.astype(np.float32) + values.astype(np.float32)).astype(np.float16)
        else:
            total = total + values
    if half:
        return (total.astype(np.float32) / np.float32(len(folds))).astype(np.float16)
    return (total / np.float32(len(folds))).astype(np.float32)


def normalized_labels(logits_cl: np.ndarray, normalizer_cl: np.ndarray) -> np.ndarray:
    """Channels-last ``(*spatial, C)`` / ``(*spatial, 1)`` -> uint16 labels, 65535 if invalid."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = (logits_cl.astype(np.float32) / normalizer_cl.astype(np.float32)).astype(np.float32)
    den = normalizer_cl[..., 0]
    invalid = ~np.isfinite(den) | (den <= 0) | ~np.isfinite(q).all(axis=-1)
    labels = np.argmax(np.where(np.isnan(q), -np.inf, q), axis=-1).astype(np.uint16)
    labels[invalid] = INVALID_LABEL
    return labels
