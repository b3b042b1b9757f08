"""NumPy float64 restatement of the reference's class-label restoration -- TEST INFRASTRUCTURE.

Follows the reference's fused device restoration and the host path it stands for:

* per-axis grid (``src/nnunet_mlx/kernels/metal_restore.py:476-495``, ``_axis_metadata``):
  target index ``t`` of an axis with source size ``S`` and target size ``T`` samples
  ``c = (t + 0.5) * (S / T) - 0.5`` in float64 (half-pixel grid), with weights
  ``(1 - f, f)``, ``f = c - floor(c)``, on source indices ``floor(c)`` and ``floor(c) + 1``;
* value (``metal_restore.py:71-139``): the sum over the eight corners, axis-0 corner
  outermost and axis 2 fastest, of ``((v * w_0) * w_1) * w_2``, rounded once to the
  logits' precision (float32, or float16 for half logits: ``ds_round_to_half``);
* label: the first class with the largest rounded value (strict ``>`` over classes);
* uncrop into a zero volume at the crop box and ``transpose(transpose_backward)``
  (``src/nnunet_mlx/prediction/export.py:363-373``).

Edges: the host path of the reference (``src/nnunet_mlx/data/resampling.py:476-502``:
skimage ``resize(order=1, mode="edge", anti_aliasing=False)``, i.e. scipy
``ndimage.zoom(order=1, mode="nearest", grid_mode=True)`` in float64, cast once to the
input dtype) clamps out-of-range source INDICES, while the Metal kernel clips the
COORDINATE into ``[0, S - 1]``.  Both put the same weight on the same voxels; they differ
only in float64 rounding at the border.  This restatement clamps indices, so its values
equal scipy's bit for bit (pinned in ``tests/test_restore_cpu.py``); the reference's own
test of the device path asserts label equality with that host path
(``tests/test_metal_restore.py:39-76``).

Only tests, ``smoke()`` and the bench CPU baseline may use this module.
"""

from __future__ import annotations

import itertools

import numpy as np


def axis_taps(source: int, target: int):
    """``(i0, i1, w0, w1)`` arrays of length ``target`` for one axis (index-clamped half-pixel grid)."""
    c = (np.arange(target, dtype=np.float64) + 0.5) * (source / target) - 0.5
    lower = np.floor(c)
    w1 = c - lower
    w0 = 1.0 - w1
    lo = lower.astype(np.int64)
    return np.clip(lo, 0, source - 1), np.clip(lo + 1, 0, source - 1), w0, w1


def resample_order1(values: np.ndarray, target) -> np.ndarray:
    """Float64 order-1 resampling of ``(C, S0, S1, S2)`` logits to ``(C, *target)`` (unrounded)."""
    target = tuple(int(t) for t in target)
    taps = [axis_taps(int(values.shape[i + 1]), target[i]) for i in range(3)]
    v = np.asarray(values).astype(np.float64)
    out = np.zeros((v.shape[0], *target), dtype=np.float64)
    shapes = ((-1, 1, 1), (1, -1, 1), (1, 1, -1))
    for corner in itertools.product((0, 1), repeat=3):
        idx = [taps[a][corner[a]].reshape(shapes[a]) for a in range(3)]
        w = [taps[a][2 + corner[a]].reshape(shapes[a]) for a in range(3)]
        out += ((v[:, idx[0], idx[1], idx[2]] * w[0]) * w[1]) * w[2]
    return out


def rounded_values(values: np.ndarray, target) -> np.ndarray:
    """Resampled values rounded once to the logits' precision (float16 for half logits, else float32)."""
    dtype = np.float16 if np.asarray(values).dtype == np.float16 else np.float32
    if tuple(values.shape[1:]) == tuple(int(t) for t in target):
        return np.asarray(values).astype(dtype)
    return resample_order1(values, target).astype(dtype)


def first_argmax(values: np.ndarray) -> np.ndarray:
    """First class with the largest value, as uint16 (strict ``>`` keeps the earliest class)."""
    best = values[0].astype(np.float32)
    labels = np.zeros(best.shape, dtype=np.uint16)
    for c in range(1, values.shape[0]):
        current = values[c].astype(np.float32)
        better = current > best
        labels[better] = c
        best = np.where(better, current, best)
    return labels


def restore_labels(values: np.ndarray, target, *, volume=None, crop_lo=(0, 0, 0), axes=(0, 1, 2)) -> np.ndarray:
    """Labels of ``(C, S0, S1, S2)`` logits resampled to ``target``, uncropped into ``volume``, permuted by ``axes``."""
    target = tuple(int(t) for t in target)
    cropped = first_argmax(rounded_values(values, target))
    volume = target if volume is None else tuple(int(v) for v in volume)
    full = np.zeros(volume, dtype=np.uint16)
    full[tuple(slice(int(lo), int(lo) + t) for lo, t in zip(crop_lo, target))] = cropped
    return np.ascontiguousarray(full.transpose(tuple(int(a) for a in axes)))
