"""Raw-case preprocessing on the GPU: the step before the sliding window.

Mirrors the reference's ``preprocess_raw_case`` (``src/nnunet_mlx/data/preprocessing.py:60-163``,
upstream ``DefaultPreprocessor.run_case_npy`` order) with the same arguments, result type and
``ContractError`` behaviour, but the volume crosses to the device once (in its own dtype) and
every pass runs there:

1. nonzero bounding box of the transposed case (``nnb_nonzero_bounds``; the plans' transpose is
   folded into the kernels' reads, no transposed copy exists), with the reference's float32
   finiteness check;
2. when a mask is needed (any scheme other than CT, or a cascade input), the nonzero mask with
   enclosed holes filled (``nnb_fill_holes_*``: 6-connected background reached from the crop
   box's faces, as scipy ``binary_fill_holes``), and the cropped previous-stage labels with -1
   outside it (``nnb_crop_labels``);
3. crop + per-channel normalisation (``nnb_crop_normalize``; CT and no-op channels in the same
   pass as the crop, z-score / rescale / RGB after float64 statistics);
4. resampling to the target spacing: upstream's torch sampling grid (``resample_torch_fornnunet``:
   ``nnb_torch_resize``, in-plane then along the separate axis when the anisotropy policy asks for
   it) for the image and the cascade labels, or the spline path for the image (below).

The result stays on the device: ``PreprocessedRawCase.data`` is a contiguous float32
``(C, *spatial)`` CUDA tensor that the predictors accept as is.

Plans that resample the image with the spline path (``resample_data_or_seg_to_shape``, nnU-Net's
default: order 3 with a separate order-0 axis for anisotropic spacing) run on the device too
(``nnb_spline_resize`` + ``nnb_nearest_axis_resize``), reproducing the reference's host path
(skimage ``resize`` = scipy ``zoom``, float64) to one float32 rounding.  Cascade labels with a
spline plan and a changed grid raise ``ContractError``.
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field

import numpy as np
import torch

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction.restore import separate_z_axis, validate_spacing

RESAMPLING_FUNCTIONS = ("resample_data_or_seg_to_shape", "resample_torch_fornnunet")
INTERPOLATION_MODES = ("linear", "nearest", "nearest-exact")
TIEBREAKS = ("nearest", "lowest", "highest")
NORMALIZATION_SCHEMES = ("CTNormalization", "ZScoreNormalization", "NoNormalization",
                         "RescaleTo01Normalization", "RGBTo01Normalization")
_TORCH_KWARGS = {"is_seg", "force_separate_z", "seg_tiebreak", "mode", "aniso_axis_mode",
                 "separate_z_anisotropy_threshold", "num_threads", "device", "memefficient_seg_resampling"}
_SPLINE_KWARGS = {"is_seg", "order", "order_z", "force_separate_z", "seg_tiebreak",
                  "separate_z_anisotropy_threshold"}
_LABEL_RANGE = (-1, 32767)


@dataclass(frozen=True)
class ResamplingContract:
    """One ``resampling_fn_*`` plan entry (reference ``src/nnunet_mlx/plans.py:32-150``)."""

    function_name: str
    order: int = 3
    order_z: int = 0
    force_separate_z: bool | None = None
    seg_tiebreak: str = "nearest"
    mode: str = "linear"
    aniso_axis_mode: str = "nearest-exact"
    separate_z_anisotropy_threshold: float = 3.0

    @classmethod
    def from_configuration(cls, configuration: Mapping[str, object], *, field: str,
                           expected_is_seg: bool) -> ResamplingContract:
        name = configuration.get(field)
        if name not in RESAMPLING_FUNCTIONS:
            raise ContractError(f"unsupported nnU-Net resampling function {name!r}")
        kwargs = configuration.get(f"{field}_kwargs", {})
        if not isinstance(kwargs, Mapping):
            raise ContractError(f"{field}_kwargs must be an object")
        torch_grid = name == "resample_torch_fornnunet"
        if bool(kwargs.get("is_seg", False)) is not expected_is_seg:
            raise ContractError(f"{field}.is_seg does not match its runtime role")
        unknown = set(kwargs) - (_TORCH_KWARGS if torch_grid else _SPLINE_KWARGS)
        if unknown:
            raise ContractError(f"{field}: unsupported kwargs: {', '.join(sorted(unknown))}")
        force = kwargs.get("force_separate_z", None if torch_grid else False)
        if force is not None and not isinstance(force, bool):
            raise ContractError(f"{field}.force_separate_z must be boolean or null")
        tiebreak = kwargs.get("seg_tiebreak", "nearest")
        if tiebreak not in TIEBREAKS:
            raise ContractError(f"{field}.seg_tiebreak must be 'nearest', 'lowest', or 'highest'")
        threshold = kwargs.get("separate_z_anisotropy_threshold", 3.0)
        if isinstance(threshold, bool) or not isinstance(threshold, int | float) or not threshold > 0:
            raise ContractError(f"{field}.separate_z_anisotropy_threshold must be positive")
        if torch_grid:
            if kwargs.get("device", "cpu") != "cpu":
                raise ContractError(f"{field}.device supports only 'cpu' host resampling")
            mode = kwargs.get("mode", "linear")
            aniso = kwargs.get("aniso_axis_mode", "nearest-exact")
            if mode not in INTERPOLATION_MODES or aniso not in INTERPOLATION_MODES:
                raise ContractError(f"{field}: unsupported interpolation mode")
            return cls(name, 1, 0, force, tiebreak, mode, aniso, float(threshold))
        order, order_z = kwargs.get("order", 3), kwargs.get("order_z", 0)
        if any(isinstance(v, bool) or not isinstance(v, int) or not 0 <= v <= 5 for v in (order, order_z)):
            raise ContractError(f"{field}: spline orders must be in [0, 5]")
        return cls(name, order, order_z, force, tiebreak, "linear", "nearest-exact", float(threshold))


@dataclass(frozen=True)
class PreprocessingPlans:
    """What preprocessing reads from a plans file for one configuration (reference ``plans.py:155-300``)."""

    transpose_forward: tuple[int, int, int]
    spacing: tuple[float | None, ...]
    normalization_schemes: tuple[str, ...]
    use_mask_for_norm: tuple[bool, ...]
    intensity_properties: dict[str, dict[str, object]] = field(default_factory=dict)
    data_resampling: ResamplingContract = ResamplingContract("resample_data_or_seg_to_shape")
    seg_resampling: ResamplingContract = ResamplingContract("resample_data_or_seg_to_shape")

    @classmethod
    def from_payload(cls, payload: Mapping[str, object], *, configuration: str) -> PreprocessingPlans:
        forward = payload.get("transpose_forward")
        if not isinstance(forward, list | tuple) or sorted(forward) != [0, 1, 2]:
            raise ContractError("transpose_forward must be a permutation of [0, 1, 2]")
        configurations = payload.get("configurations")
        if not isinstance(configurations, Mapping) or not isinstance(configurations.get(configuration), Mapping):
            raise ContractError(f"plans have no configuration {configuration!r}")
        config = configurations[configuration]
        spacing = config.get("spacing")
        if not isinstance(spacing, list | tuple) or len(spacing) not in (2, 3):
            raise ContractError("configuration spacing must have two or three entries")
        schemes = tuple(config.get("normalization_schemes") or ())
        masks = tuple(bool(v) for v in config.get("use_mask_for_norm") or ())
        if not schemes or len(masks) != len(schemes):
            raise ContractError("normalization_schemes and use_mask_for_norm must match per channel")
        intensity = payload.get("foreground_intensity_properties_per_channel",
                                payload.get("foreground_intensity_properties_by_modality", {}))
        return cls(
            transpose_forward=tuple(int(a) for a in forward),  # type: ignore[arg-type]
            spacing=tuple(None if v is None else float(v) for v in spacing),
            normalization_schemes=schemes,
            use_mask_for_norm=masks,
            intensity_properties=dict(intensity) if isinstance(intensity, Mapping) else {},
            data_resampling=ResamplingContract.from_configuration(config, field="resampling_fn_data",
                                                                  expected_is_seg=False),
            seg_resampling=ResamplingContract.from_configuration(config, field="resampling_fn_seg",
                                                                 expected_is_seg=True),
        )


@dataclass(frozen=True)
class PreprocessedRawCase:
    """Preprocessed case (reference ``preprocessing.py:29-43``): ``data`` (C, X, Y, Z) float32 on the device."""

    data: torch.Tensor
    previous_stage: torch.Tensor | None
    properties: dict[str, object]


def compute_new_shape(old_shape: Sequence[int], old_spacing: Sequence[float],
                      new_spacing: Sequence[float]) -> tuple[int, ...]:
    """``round(size * old / new)`` per axis with Python rounding (reference ``resampling.py:46-69``)."""
    if not (len(old_shape) == len(old_spacing) == len(new_spacing) and len(old_shape) in (2, 3)):
        raise ContractError("shape and spacing ranks must match in 2-D or 3-D")
    if any(s < 1 for s in old_shape) or any(not math.isfinite(v) or v <= 0 for v in (*old_spacing, *new_spacing)):
        raise ContractError("resampling shape and spacing values must be positive")
    return tuple(round(o / n * s) for o, n, s in zip(old_spacing, new_spacing, old_shape, strict=True))


def _number(value: object, name: str) -> float:
    if isinstance(value, bool) or not isinstance(value, int | float) or not math.isfinite(float(value)):
        raise ContractError(f"{name} must be a finite number")
    return float(value)


def _channel_normalizations(plans: PreprocessingPlans, channels: int) -> list[kernels.ChannelNormalization]:
    """Per-channel kernel parameters; CT scalars rounded to float32 as NumPy rounds Python floats."""
    if len(plans.normalization_schemes) != channels:
        raise ContractError("normalization schemes do not match the input channels")
    result = []
    for c, scheme in enumerate(plans.normalization_schemes):
        if scheme not in NORMALIZATION_SCHEMES:
            raise ContractError(f"unsupported nnU-Net normalization scheme {scheme!r}")
        if scheme != "CTNormalization":
            result.append(kernels.ChannelNormalization(scheme, bool(plans.use_mask_for_norm[c])))
            continue
        stats = plans.intensity_properties.get(str(c), {})
        mean = _number(stats.get("mean"), "CT mean")
        std = _number(stats.get("std"), "CT std")
        if std <= 0:
            raise ContractError("CT std must be positive")
        lower = _number(stats.get("percentile_00_5"), "CT lower percentile")
        upper = _number(stats.get("percentile_99_5"), "CT upper percentile")
        if lower > upper:
            raise ContractError("CT intensity percentiles are reversed")
        f32 = lambda v: float(np.float32(v))  # noqa: E731
        result.append(kernels.ChannelNormalization(scheme, False, f32(lower), f32(upper), f32(mean),
                                                   f32(max(std, 1e-8))))
    return result


def _upload(values: np.ndarray | torch.Tensor, device: torch.device) -> torch.Tensor:
    if isinstance(values, torch.Tensor):
        return values.to(device).contiguous()
    host = torch.from_numpy(np.ascontiguousarray(values))
    if host.numel() * host.element_size() >= (1 << 20):
        host = host.pin_memory()
    return host.to(device, non_blocking=True)


_DEVICE_DTYPES = {np.dtype(t) for t in ("float32", "float64", "int16", "uint8", "uint16", "int32")}


def resample_torch_device(values: torch.Tensor, new_shape: Sequence[int], current_spacing: Sequence[float],
                          new_spacing: Sequence[float], contract: ResamplingContract, *,
                          is_seg: bool) -> torch.Tensor:
    """Torch-grid resampling of device ``(C, X, Y, Z)`` float32 values or int32 labels.

    Reference ``data/resampling.py:87-172`` / ``175-244`` with ``metal_torch_resample.py:196-216``:
    equal shapes return the input; otherwise, when the anisotropy policy names a separate
    axis, the in-plane axes are resampled first (that axis kept) and then that axis with the
    plan's ``aniso_axis_mode``.  Labels are decided between the passes.
    """
    target = tuple(int(v) for v in new_shape)
    if len(target) != 3 or min(target) < 1:
        raise ContractError("resampling target shape must be positive")
    current = validate_spacing(current_spacing, name="current spacing")
    new = validate_spacing(new_spacing, name="new spacing")
    if tuple(values.shape[1:]) == target:
        return values.contiguous()
    _, axis = separate_z_axis(current, new, force=contract.force_separate_z,
                              threshold=contract.separate_z_anisotropy_threshold)
    if axis is None:
        return kernels.torch_resize(values, target, contract.mode, labels=is_seg, tiebreak=contract.seg_tiebreak)
    in_plane = tuple(target[i] if i != axis else int(values.shape[1 + i]) for i in range(3))
    # a pass whose source already has its target shape is the identity (metal_torch_resample.py:172-173)
    first = values if tuple(values.shape[1:]) == in_plane else kernels.torch_resize(
        values, in_plane, contract.mode, labels=is_seg, tiebreak=contract.seg_tiebreak)
    if tuple(first.shape[1:]) == target:
        return first.contiguous()
    return kernels.torch_resize(first, target, contract.aniso_axis_mode, labels=is_seg,
                                tiebreak=contract.seg_tiebreak)


def resample_spline_device(values: torch.Tensor, new_shape: Sequence[int], current_spacing: Sequence[float],
                           new_spacing: Sequence[float], contract: ResamplingContract) -> torch.Tensor:
    """Spline resampling of device ``(C, X, Y, Z)`` float32 image values (``resample_data_or_seg_to_shape``).

    Reference ``data/resampling.py:87-172`` (host path: skimage ``resize`` = scipy ``zoom(order,
    mode="nearest", grid_mode=True)`` per channel, float64 arithmetic, one rounding to float32): without a
    separate axis every axis is resampled at ``order``; with one (``separate_z_axis``) the other two are
    resampled plane by plane into a float64 intermediate (``:268-306``), then that axis at ``order_z``
    (0: half-pixel nearest indices, ``:379-427``) and the result rounded once.  Orders 1 and 3 and
    ``order_z`` 0 (nnU-Net's defaults are 3 and 0) run on the device; others raise ``ContractError``.
    """
    target = tuple(int(v) for v in new_shape)
    if len(target) != 3 or min(target) < 1:
        raise ContractError("resampling target shape must be positive")
    current = validate_spacing(current_spacing, name="current spacing")
    new = validate_spacing(new_spacing, name="new spacing")
    if tuple(values.shape[1:]) == target:
        return values.contiguous()
    if contract.order not in (1, 3):
        raise ContractError(f"device preprocessing supports spline orders 1 and 3, not {contract.order}")
    separate, axis = separate_z_axis(current, new, force=contract.force_separate_z,
                                     threshold=contract.separate_z_anisotropy_threshold)
    if not separate or axis is None:
        return kernels.spline_resize(values, target, axes=7, order=contract.order)
    intermediate_shape = tuple(target[i] if i != axis else int(values.shape[1 + i]) for i in range(3))
    intermediate = kernels.spline_resize(values, intermediate_shape, axes=7 & ~(1 << axis), order=contract.order,
                                         float64_out=True)
    if intermediate_shape != target and contract.order_z != 0:
        raise ContractError(f"device preprocessing supports out-of-plane order 0, not {contract.order_z}")
    return kernels.nearest_axis_resize(intermediate, target)


def crop_to_nonzero_device(raw: torch.Tensor, transpose: Sequence[int], previous: torch.Tensor | None, *,
                           mask_required: bool):
    """Device ``crop_to_nonzero`` of the transposed raw case (reference ``preprocessing.py:166-217``).

    Returns ``(box_lo, box_dims, state, cropped_previous, bounds)``: the crop box in plans order,
    the int8 hole-filled mask state of the box (``None`` without ``mask_required``; inside is
    ``state != 2``), the cropped int32 previous stage with -1 outside the mask (or ``None``) and
    the half-open ``(start, stop)`` bounds.  One synchronisation reads the bounds.
    """
    bounds = kernels.to_host(kernels.nonzero_bounds(raw, transpose))
    if int(bounds[6]) != 0:
        raise ContractError("raw nnU-Net cases must remain finite after float32 conversion")
    lo, hi = [int(v) for v in bounds[:3]], [int(v) for v in bounds[3:6]]
    if hi[0] < 0:
        raise ContractError("raw nnU-Net case has no nonzero voxels")
    dims = [h - l + 1 for l, h in zip(lo, hi, strict=True)]
    state = kernels.fill_holes(raw, transpose, lo, dims) if mask_required else None
    cropped_previous = None
    if previous is not None:
        cropped_previous = kernels.crop_labels(previous, raw, transpose, lo, dims, state)
    return lo, dims, state, cropped_previous, tuple((l, l + d) for l, d in zip(lo, dims, strict=True))


def preprocess_raw_case(data: np.ndarray | torch.Tensor, properties: Mapping[str, object],
                        plans: PreprocessingPlans, *, segmentation_previous_stage=None,
                        device: torch.device | str | None = None) -> PreprocessedRawCase:
    """Transpose, nonzero crop, normalisation and torch-grid resampling of one raw case on the GPU.

    Same contract as the reference's ``preprocess_raw_case`` (``preprocessing.py:60-163``):
    ``data`` is ``(C, X, Y, Z)`` real numbers in the image's axis order, ``properties["spacing"]``
    three positive voxel sizes in that order; ``segmentation_previous_stage`` is an optional
    ``(1, X, Y, Z)`` non-negative integer cascade input.  The returned properties add
    ``shape_before_cropping``, ``bbox_used_for_cropping`` and
    ``shape_after_cropping_and_before_resampling`` (plans axis order).
    """
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    values = data if isinstance(data, torch.Tensor) else np.asarray(data)
    if values.ndim != 4 or int(values.shape[0]) < 1:
        raise ContractError("raw nnU-Net cases must have CXYZ layout")
    dtype = np.dtype(str(values.dtype).removeprefix("torch.")) if isinstance(values, torch.Tensor) else values.dtype
    if dtype.kind not in "iuf":
        raise ContractError("raw nnU-Net cases must contain finite real numeric values")
    if dtype not in _DEVICE_DTYPES:
        # other integer widths and float16 convert exactly to float32 before upload
        values = np.asarray(values.cpu() if isinstance(values, torch.Tensor) else values).astype(np.float32)
    channels = int(values.shape[0])
    norms = _channel_normalizations(plans, channels)
    result_properties = dict(properties)
    spacing = result_properties.get("spacing")
    if not isinstance(spacing, list | tuple) or len(spacing) != 3:
        raise ContractError("raw medical-image spacing must contain three values")
    spacing = validate_spacing(spacing, name="image spacing")
    previous = None
    if segmentation_previous_stage is not None:
        labels = np.asarray(segmentation_previous_stage.cpu() if isinstance(segmentation_previous_stage, torch.Tensor)
                            else segmentation_previous_stage)
        if labels.shape != (1, *values.shape[1:]):
            raise ContractError("previous-stage segmentation shape does not match the image")
        if not np.issubdtype(labels.dtype, np.integer):
            raise ContractError("previous-stage segmentation must contain integer labels")
        if labels.size and (labels.min() < 0 or labels.max() > np.iinfo(np.int32).max):
            raise ContractError("raw previous-stage segmentation labels must be non-negative int32 values")
        previous = _upload(labels.astype(np.int32), device)
    raw = _upload(values, device)
    transpose = plans.transpose_forward
    original_spacing = tuple(spacing[a] for a in transpose)
    result_properties["shape_before_cropping"] = tuple(int(values.shape[1 + a]) for a in transpose)
    mask_required = previous is not None or any(s != "CTNormalization" for s in plans.normalization_schemes)
    lo, dims, state, cropped_previous, bounds = crop_to_nonzero_device(raw, transpose, previous,
                                                                      mask_required=mask_required)
    result_properties["bbox_used_for_cropping"] = [list(pair) for pair in bounds]
    result_properties["shape_after_cropping_and_before_resampling"] = tuple(dims)
    normalized, errors = kernels.crop_normalize(raw, transpose, lo, dims, norms, state=state,
                                                labels=cropped_previous)
    counts = kernels.to_host(errors)
    if int(counts[2]):
        raise ContractError("z-score normalization mask is empty")
    if int(counts[1]):
        raise ContractError("RGB normalization requires values in [0, 255]")
    if int(counts[0]):
        raise ContractError("normalization produced non-finite values")
    configured = tuple(plans.spacing)
    if len(configured) != 3:
        configured = (original_spacing[0], *configured)
    target_spacing = tuple(o if c is None else float(c) for c, o in zip(configured, original_spacing, strict=True))
    new_shape = compute_new_shape(tuple(dims), original_spacing, target_spacing)
    if min(new_shape) < 1:
        raise ContractError("resampling target shape must be positive")
    changed = tuple(new_shape) != tuple(dims)
    if changed and cropped_previous is not None and plans.seg_resampling.function_name != "resample_torch_fornnunet":
        raise ContractError("device preprocessing resamples cascade labels on the torch grid only "
                            f"({plans.seg_resampling.function_name} with a changed grid is not supported)")
    if plans.data_resampling.function_name == "resample_torch_fornnunet":
        resampled = resample_torch_device(normalized, new_shape, original_spacing, target_spacing,
                                          plans.data_resampling, is_seg=False)
    else:
        resampled = resample_spline_device(normalized, new_shape, original_spacing, target_spacing,
                                           plans.data_resampling)
    resampled_previous = None
    if cropped_previous is not None:
        if plans.seg_resampling.function_name == "resample_torch_fornnunet" and (
                int(torch.amin(cropped_previous)) < _LABEL_RANGE[0]
                or int(torch.amax(cropped_previous)) > _LABEL_RANGE[1]):
            raise ContractError("resample_torch_fornnunet labels must be in [-1, 32767]")
        resampled_previous = resample_torch_device(cropped_previous, new_shape, original_spacing, target_spacing,
                                                   plans.seg_resampling, is_seg=True)
    return PreprocessedRawCase(resampled, resampled_previous, result_properties)
