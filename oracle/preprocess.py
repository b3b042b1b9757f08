"""NumPy restatement of the reference's raw-case preprocessing -- TEST INFRASTRUCTURE.

Follows the reference's ``preprocess_raw_case`` (``src/nnunet_mlx/data/preprocessing.py:60-163``)
for plans that resample with the torch sampling grid (``resample_torch_fornnunet``) or keep
the grid, in upstream's step order: transpose by ``transpose_forward``, crop to the nonzero
bounding box, normalise each channel, resample to the target spacing.

* crop (``preprocessing.py:166-217``): mask = any channel nonzero, holes filled (scipy
  ``binary_fill_holes``, as the reference resolves it at ``preprocessing.py:340-343``) when a
  mask is needed; bounds are the mask's per-axis extent; the int8 segmentation mask is 0
  inside and -1 outside the filled region; previous-stage background outside it becomes -1.
* normalisation (``preprocessing.py:222-319``): CT clip/shift/scale, z-score (over the mask
  when ``use_mask_for_norm``), rescale to [0, 1], RGB / 255, none -- float32 arithmetic with
  the scalars rounded to float32 as NumPy does for Python floats.
* spline resampling (the reference's host path, ``src/nnunet_mlx/data/resampling.py:87-172,268-306,379-427``):
  skimage ``resize(order, mode="edge", anti_aliasing=False)`` per channel, which is scipy
  ``ndimage.zoom(order, mode="nearest", grid_mode=True)`` (skimage is absent here; scipy is the
  reference's own dependency that does the arithmetic), with the separate-axis planes kept in float64
  and the out-of-plane axis taken at half-pixel nearest indices;
* torch-grid resampling (``src/nnunet_mlx/kernels/metal_torch_resample.py:51-131``, its
  separate-axis composition ``:196-216`` and the policy of
  ``src/nnunet_mlx/data/resampling.py:87-172,175-244,587-614``): per axis ``scale =
  float32(source / target)``; nearest index ``min(int(scale * (t + s)), S - 1)`` with ``s`` =
  0 ("nearest") or 0.5 ("nearest-exact", and the linear mode's nearest label); linear
  coordinate ``max(scale * (t + 0.5) - 0.5, 0)`` in float32 (no contraction), lower index
  clamped, upper ``min(lower + 1, S - 1)``, weights ``(1 - f, f)``; image value = float64 sum
  over the eight corners (axis 0 outermost) of ``((v * w_0) * w_1) * w_2`` rounded once to
  float32; labels score each distinct corner label by the summed ``1000 * w_0 * w_1 * w_2``
  of its corners, rounded float64 -> float32 -> float16, and keep the best score with the
  plan's tie rule (lowest, highest, or nearest-neighbour label then lowest).

The reference computes the products in double-single arithmetic; float64 has more precision,
so both round to the same float32 except in cases this restatement's golden tests would show
(``tests/test_preprocess_cpu.py`` pins it against upstream's recorded label resampling and
against ``torch.nn.functional.interpolate``).

Only tests, ``smoke()`` and the bench CPU baseline may use this module.
"""

from __future__ import annotations

import itertools

import numpy as np

MODES = ("linear", "nearest", "nearest-exact")
TIEBREAKS = ("lowest", "highest", "nearest")


def _axis(source: int, target: int, mode: str):
    """Per-target-index (nearest, lower, upper, w0, w1) of one axis, float32 coordinates."""
    scale = np.float32(source / target)
    t = np.arange(target, dtype=np.float32)
    shift = np.float32(0.0 if mode == "nearest" else 0.5)
    scaled = (scale * (t + shift)).astype(np.float32)
    nearest = np.minimum(scaled.astype(np.int64), source - 1)
    coordinate = np.maximum((scale * (t + np.float32(0.5))).astype(np.float32) - np.float32(0.5),
                            np.float32(0)).astype(np.float32)
    lower = np.minimum(coordinate.astype(np.int64), source - 1)
    upper = np.minimum(lower + 1, source - 1)
    fraction = (coordinate - np.floor(coordinate)).astype(np.float32)
    w1 = fraction.astype(np.float64)
    w0 = 1.0 - w1
    return nearest, lower, upper, w0, w1


def torch_resize(data: np.ndarray, shape, mode: str, *, is_seg: bool, tiebreak: str = "nearest") -> np.ndarray:
    """One torch-grid pass over ``(C, S0, S1, S2)``; output has the input's dtype."""
    values = np.asarray(data)
    shape = tuple(int(v) for v in shape)
    if values.shape[1:] == shape:
        return values.copy()
    axes = [_axis(int(s), int(t), mode) for s, t in zip(values.shape[1:], shape, strict=True)]
    if mode != "linear":
        n0, n1, n2 = (a[0] for a in axes)
        return values[:, n0[:, None, None], n1[None, :, None], n2[None, None, :]].copy()
    corners = []
    for bits in itertools.product((0, 1), repeat=3):
        idx = [a[2] if b else a[1] for a, b in zip(axes, bits, strict=True)]
        w = [a[4] if b else a[3] for a, b in zip(axes, bits, strict=True)]
        sample = values[:, idx[0][:, None, None], idx[1][None, :, None], idx[2][None, None, :]]
        corners.append((sample, w))
    if not is_seg:
        total = np.zeros((values.shape[0], *shape), dtype=np.float64)
        for sample, w in corners:
            term = sample.astype(np.float64) * w[0][:, None, None]
            term = term * w[1][None, :, None]
            term = term * w[2][None, None, :]
            total = total + term
        return total.astype(np.float32)
    weights = []
    for _, w in corners:
        term = np.float64(1000.0) * w[0][:, None, None]
        term = term * w[1][None, :, None]
        term = term * w[2][None, None, :]
        weights.append(np.broadcast_to(term, (values.shape[0], *shape)))
    samples = [s.astype(np.int64) for s, _ in corners]
    n0, n1, n2 = (a[0] for a in axes)
    nearest_label = values[:, n0[:, None, None], n1[None, :, None], n2[None, None, :]].astype(np.int64)
    best = np.full((values.shape[0], *shape), -1.0, dtype=np.float32)
    winner = np.zeros((values.shape[0], *shape), dtype=np.int64)
    for c in range(8):
        label = samples[c]
        seen = np.zeros(label.shape, dtype=bool)
        for p in range(c):
            seen |= samples[p] == label
        score = np.zeros(label.shape, dtype=np.float64)
        for k in range(8):
            score = score + np.where(samples[k] == label, weights[k], 0.0)
        rounded = score.astype(np.float32).astype(np.float16).astype(np.float32)
        if tiebreak == "lowest":
            preferred = label < winner
        elif tiebreak == "highest":
            preferred = label > winner
        else:
            preferred = (label == nearest_label) | ((winner != nearest_label) & (label < winner))
        take = ~seen & ((rounded > best) | ((rounded == best) & preferred))
        best = np.where(take, rounded, best)
        winner = np.where(take, label, winner)
    return winner.astype(values.dtype)


def separate_z_axis(current, new, *, force, threshold: float = 3.0):
    """Unique coarsest axis for separate resampling (reference ``data/resampling.py:587-614``)."""
    if force is None:
        current_aniso = max(current) / min(current) > threshold
        separate = current_aniso or max(new) / min(new) > threshold
        basis = current if current_aniso else new
    else:
        separate = bool(force)
        basis = current
    if not separate:
        return False, None
    largest = max(basis)
    axes = [i for i, s in enumerate(basis) if largest / s == 1]
    return (True, axes[0]) if len(axes) == 1 else (False, None)


def resample_torch(data: np.ndarray, shape, current, new, *, mode="linear", aniso_axis_mode="nearest-exact",
                   force_separate_z=None, threshold=3.0, is_seg=False, tiebreak="nearest") -> np.ndarray:
    """Torch-grid resampling with the plan's separate-axis policy (in-plane pass, then the axis)."""
    values = np.asarray(data)
    shape = tuple(int(v) for v in shape)
    if values.shape[1:] == shape:
        return values.copy()
    _, axis = separate_z_axis(current, new, force=force_separate_z, threshold=threshold)
    if axis is None:
        return torch_resize(values, shape, mode, is_seg=is_seg, tiebreak=tiebreak)
    in_plane = tuple(shape[i] if i != axis else values.shape[1 + i] for i in range(3))
    first = torch_resize(values, in_plane, mode, is_seg=is_seg, tiebreak=tiebreak)
    return torch_resize(first, shape, aniso_axis_mode, is_seg=is_seg, tiebreak=tiebreak)


def nearest_axis_indices(old: int, new: int) -> np.ndarray:
    """Half-pixel nearest indices of one resized axis (reference ``data/resampling.py:401-407``)."""
    coordinates = float(old) / new * (np.arange(new, dtype=np.float64) + 0.5) - 0.5
    return np.clip(np.floor(coordinates + 0.5).astype(np.intp), 0, old - 1)


def _zoom(values: np.ndarray, shape, order: int) -> np.ndarray:
    """skimage ``resize(order, mode="edge", anti_aliasing=False)`` as scipy ``zoom`` (grid mode, "nearest")."""
    from scipy import ndimage

    out = ndimage.zoom(values, np.divide(shape, values.shape), order=order, mode="nearest", grid_mode=True)
    assert out.shape == tuple(shape)
    return out


def resample_spline(values: np.ndarray, new_shape, current, new, *, order=3, order_z=0, force_separate_z=False,
                    threshold=3.0) -> np.ndarray:
    """Spline resampling of float32 ``(C, X, Y, Z)`` data (reference ``data/resampling.py:87-172,268-306``)."""
    values = np.asarray(values, dtype=np.float32)
    shape = tuple(int(v) for v in new_shape)
    if values.shape[1:] == shape:
        return values.copy()
    _, axis = separate_z_axis(current, new, force=force_separate_z, threshold=threshold)
    if axis is None:
        return np.stack([_zoom(channel, shape, order) for channel in values]).astype(np.float32)
    plane_shape = tuple(shape[i] for i in range(3) if i != axis)
    result = []
    for channel in values:
        planes = [_zoom(np.take(channel, k, axis=axis).astype(np.float64), plane_shape, order)
                  for k in range(channel.shape[axis])]
        intermediate = np.stack(planes, axis=axis)
        if intermediate.shape != shape:
            assert order_z == 0
            intermediate = np.take(intermediate, nearest_axis_indices(intermediate.shape[axis], shape[axis]),
                                   axis=axis)
        result.append(intermediate.astype(np.float32))
    return np.stack(result)


def crop_to_nonzero(data: np.ndarray, previous: np.ndarray | None, *, mask_required: bool):
    """(cropped float32 data, int8 mask, cropped previous or None, bounds) as the reference returns."""
    from scipy.ndimage import binary_fill_holes

    mask = np.any(data != 0, axis=0)
    if mask_required:
        mask = binary_fill_holes(mask)
    projections = [np.flatnonzero(np.any(mask, axis=tuple(o for o in range(3) if o != a))) for a in range(3)]
    if not projections[0].size:
        raise ValueError("no nonzero voxels")
    bounds = tuple((int(p[0]), int(p[-1]) + 1) for p in projections)
    slices = tuple(slice(a, b) for a, b in bounds)
    cropped = np.ascontiguousarray(data[(slice(None), *slices)], dtype=np.float32)
    inside = mask[slices]
    seg = (np.where(inside, np.int8(0), np.int8(-1))[None] if mask_required
           else np.zeros((1, *cropped.shape[1:]), dtype=np.int8))
    cropped_previous = None
    if previous is not None:
        cropped_previous = np.array(previous[(slice(None), *slices)], copy=True)
        cropped_previous[(cropped_previous == 0) & ~inside[None]] = -1
    return cropped, seg, cropped_previous, bounds


def normalize_channel(image: np.ndarray, mask: np.ndarray, *, scheme: str, use_mask: bool,
                      intensity: dict) -> np.ndarray:
    """One channel's plans normalisation in float32 (reference ``preprocessing.py:272-319``)."""
    result = np.asarray(image, dtype=np.float32).copy()
    if scheme == "CTNormalization":
        np.clip(result, float(intensity["percentile_00_5"]), float(intensity["percentile_99_5"]), out=result)
        result -= float(intensity["mean"])
        result /= max(float(intensity["std"]), 1e-8)
        return result
    if scheme == "ZScoreNormalization":
        selected_mask = mask >= 0 if use_mask else np.ones(result.shape, dtype=bool)
        selected = result[selected_mask]
        mean = float(selected.mean())
        std = float(selected.std())
        result[selected_mask] = (result[selected_mask] - mean) / max(std, 1e-8)
        return result
    if scheme == "NoNormalization":
        return result
    if scheme == "RescaleTo01Normalization":
        result -= float(result.min())
        result /= max(float(result.max()), 1e-8)
        return result
    if scheme == "RGBTo01Normalization":
        result /= 255
        return result
    raise ValueError(scheme)


def compute_new_shape(old_shape, old_spacing, new_spacing):
    """``round(size * old / new)`` per axis with Python rounding (reference ``resampling.py:46-69``)."""
    return tuple(round(o / n * s) for o, n, s in zip(old_spacing, new_spacing, old_shape, strict=True))


def preprocess(data: np.ndarray, spacing, *, transpose_forward, configured_spacing, schemes, use_mask,
               intensities, data_resampling: dict, seg_resampling: dict, previous: np.ndarray | None = None):
    """(data, previous, properties) of the reference's ``preprocess_raw_case`` for torch-grid plans."""
    transpose = (0, *(a + 1 for a in transpose_forward))
    values = np.asarray(data).transpose(transpose).astype(np.float32)
    prev = None if previous is None else np.asarray(previous).transpose(transpose)
    original = tuple(float(spacing[a]) for a in transpose_forward)
    mask_required = prev is not None or any(s != "CTNormalization" for s in schemes)
    cropped, mask, cropped_prev, bounds = crop_to_nonzero(values, prev, mask_required=mask_required)
    norm_mask = mask if cropped_prev is None else cropped_prev
    normalized = cropped.copy()
    for c, scheme in enumerate(schemes):
        normalized[c] = normalize_channel(normalized[c], norm_mask[0], scheme=scheme, use_mask=use_mask[c],
                                          intensity=intensities.get(str(c), {}))
    configured = tuple(configured_spacing)
    if len(configured) != 3:
        configured = (original[0], *configured)
    target = tuple(o if c is None else float(c) for c, o in zip(configured, original, strict=True))
    new_shape = compute_new_shape(normalized.shape[1:], original, target)
    if data_resampling.get("spline"):
        spline = {k: v for k, v in data_resampling.items() if k != "spline"}
        out = resample_spline(normalized, new_shape, original, target, **spline)
    else:
        out = resample_torch(normalized, new_shape, original, target, is_seg=False, **data_resampling)
    out_prev = None if cropped_prev is None else resample_torch(cropped_prev, new_shape, original, target,
                                                                is_seg=True, **seg_resampling)
    properties = {"shape_before_cropping": tuple(values.shape[1:]),
                  "bbox_used_for_cropping": [list(b) for b in bounds],
                  "shape_after_cropping_and_before_resampling": tuple(cropped.shape[1:])}
    return out, out_prev, properties
