"""Device restoration of class labels: the step after the sliding window.

Class logits on the network's grid are resampled to the cropped original
grid, reduced to first-argmax labels, placed into the uncropped volume and
put back into the image's axis order, all in one CUDA kernel
(``nnb_restore_class_labels``); only the final uint16 volume crosses to the
host.  Mirrors the reference's fused restoration API
(``src/nnunet_mlx/kernels/metal_restore.py:292-401``) and its export-level
callers (``src/nnunet_mlx/prediction/export.py:305-373``), with the same
support rules and ``ContractError`` behaviour:

* supported: order-1 ``resample_data_or_seg_to_shape`` plans without separate-axis
  resampling, or equal source and target grids (argmax only, any policy);
* everything else returns ``None`` / ``False`` so that the caller takes its host path.

Interpolation is the host spline path's at order 1 (float64, half-pixel grid,
edge-clamped indices, one rounding to the logits' dtype), reproduced operation
for operation, so the labels equal the host path's.  Unlike the Metal kernel
(double-single arithmetic) there is no magnitude limit: any finite float32 or
float16 logits are accepted; non-finite interpolated values raise.
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import dataclass

import numpy as np
import torch

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError

ANISOTROPY_THRESHOLD = 3.0
MAXIMUM_CLASSES = 65536
_INT32_MAX = 2**31 - 1


@dataclass(frozen=True)
class ResamplingContract:
    """The plans' probability-resampling entry (reference ``src/nnunet_mlx/plans.py:32-58``)."""

    function_name: str
    order: int
    order_z: int
    force_separate_z: bool | None
    separate_z_anisotropy_threshold: float = ANISOTROPY_THRESHOLD


@dataclass(frozen=True)
class ConfigurationContract:
    """The parts of a plans configuration restoration reads: target spacing and resampling policy."""

    spacing: tuple[float | None, ...]
    probability_resampling: ResamplingContract


@dataclass(frozen=True)
class PlansContract:
    """Axis order of the plans (``transpose_backward`` inverts ``transpose_forward``) and one configuration."""

    transpose_forward: tuple[int, int, int]
    transpose_backward: tuple[int, int, int]
    configuration: ConfigurationContract


@dataclass(frozen=True)
class LabelSemantics:
    """Network output channels and whether they are regions (reference ``data/labels.py:25``)."""

    output_channels: int
    has_regions: bool = False


@dataclass(frozen=True)
class RestoredPrediction:
    """Labels in the image's own grid and axis order (reference ``prediction/export.py:58-70``)."""

    segmentation: np.ndarray
    probabilities: np.ndarray | None = None


def validate_spacing(value: Sequence[float], *, name: str) -> tuple[float, float, float]:
    """Three finite positive spacings (reference ``data/resampling.py:617-622``)."""
    try:
        result = tuple(float(item) for item in value if not isinstance(item, bool))
    except (TypeError, ValueError) as error:
        raise ContractError(f"{name} must contain three positive values") from error
    if len(result) != 3 or len(result) != len(tuple(value)) or any(not math.isfinite(v) or v <= 0 for v in result):
        raise ContractError(f"{name} must contain three positive values")
    return result  # type: ignore[return-value]


def separate_z_axis(current_spacing, new_spacing, *, force: bool | None,
                    threshold: float = ANISOTROPY_THRESHOLD) -> tuple[bool, int | None]:
    """Whether one coarse axis is resampled on its own, and which (upstream nnU-Net's policy).

    The spacing that decides is chosen first: with ``force=True`` the current
    spacing, with ``force=False`` none; with ``force=None`` the first of the
    current and the target spacing whose largest/smallest ratio exceeds
    ``threshold``.  The separate axis is that spacing's unique coarsest axis; a
    tie for the coarsest spacing means no separate axis (reference
    ``data/resampling.py:587-616``, pinned against the reference's own decisions).
    """
    def exceeds(spacing) -> bool:
        return max(spacing) / min(spacing) > threshold

    if force is None:
        deciding = next((sp for sp in (current_spacing, new_spacing) if exceeds(sp)), None)
    else:
        deciding = current_spacing if force else None
    if deciding is None:
        return False, None
    coarsest = [axis for axis, value in enumerate(deciding) if value == max(deciding)]
    return (True, coarsest[0]) if len(coarsest) == 1 else (False, None)


def _target_shape(new_shape: Sequence[int]) -> tuple[int, int, int]:
    result = tuple(int(v) for v in new_shape)
    if len(result) != 3 or any(v < 1 for v in result):
        raise ContractError("restoration target shape must contain three positive values")
    return result  # type: ignore[return-value]


def _validate_index_range(dims: Sequence[int], target: Sequence[int]) -> None:
    if any(int(v) > _INT32_MAX for v in (*dims, *target)):
        raise ContractError("restoration dimensions exceed the int32 range")


def device_class_restore_supported(source_shape: Sequence[int], new_shape: Sequence[int],
                                   current_spacing: Sequence[float], new_spacing: Sequence[float],
                                   contract: ResamplingContract, *, classes: int) -> bool:
    """Whether the device kernel covers this geometry and policy (reference ``metal_restore.py:336-360``)."""
    target = _target_shape(new_shape)
    if len(source_shape) != 3 or classes < 1 or classes > MAXIMUM_CLASSES:
        return False
    _validate_index_range((classes, *source_shape), target)
    if tuple(int(v) for v in source_shape) == target:
        return True
    if contract.function_name != "resample_data_or_seg_to_shape" or contract.order != 1:
        return False
    separate, _ = separate_z_axis(validate_spacing(current_spacing, name="current spacing"),
                                  validate_spacing(new_spacing, name="new spacing"),
                                  force=contract.force_separate_z,
                                  threshold=contract.separate_z_anisotropy_threshold)
    return not separate


def restore_labels_on_device(logits: torch.Tensor, new_shape: Sequence[int], *, class_axis: int = 0,
                             volume_shape: Sequence[int] | None = None, crop_lo: Sequence[int] = (0, 0, 0),
                             axes: Sequence[int] = (0, 1, 2), label_dtype: torch.dtype = torch.uint16
                             ) -> torch.Tensor:
    """Device labels of CUDA class logits: resample to ``new_shape``, argmax, uncrop, permute.

    The result stays on the device (``volume_shape`` permuted by ``axes``); a
    non-finite interpolated value raises ``ContractError`` (one synchronisation).
    """
    labels, invalid = kernels.restore_class_labels(logits, _target_shape(new_shape), class_axis=class_axis,
                                                   volume=volume_shape, crop_lo=crop_lo, axes=axes,
                                                   label_dtype=label_dtype)
    if int(invalid.item()) != 0:
        raise ContractError("class-logit restoration produced non-finite values")
    return labels


def resample_class_logits_argmax_device(logits: np.ndarray, new_shape: Sequence[int]) -> np.ndarray:
    """Host ``(C, X, Y, Z)`` float32/float16 logits -> uint16 labels on ``new_shape`` via the GPU.

    Counterpart of the reference's ``resample_class_logits_argmax_metal``
    (``metal_restore.py:292-324``): no spacing or separate-axis policy is applied;
    ties go to the first class; half logits are rounded to half after interpolation.
    """
    values = np.asarray(logits)
    target = _target_shape(new_shape)
    if (values.ndim != 4 or int(values.shape[0]) < 1 or any(int(v) < 1 for v in values.shape[1:])
            or values.dtype not in (np.dtype(np.float32), np.dtype(np.float16))):
        raise ContractError("device restoration requires non-empty float32 or float16 CXYZ logits")
    if int(values.shape[0]) > MAXIMUM_CLASSES:
        raise ContractError("device restoration exceeds the uint16 label range")
    if not np.isfinite(values).all():
        raise ContractError("device restoration requires finite logits")
    _validate_index_range(values.shape, target)
    device = torch.device("cuda", torch.cuda.current_device())
    host = torch.from_numpy(np.ascontiguousarray(values))
    staged = host.pin_memory() if host.numel() * host.element_size() >= (1 << 20) else host
    on_device = staged.to(device, non_blocking=True)
    return kernels.to_host(restore_labels_on_device(on_device, target, class_axis=0))


def resample_device_logits_argmax(logits: torch.Tensor, new_shape: Sequence[int], current_spacing: Sequence[float],
                                  new_spacing: Sequence[float], contract: ResamplingContract) -> np.ndarray | None:
    """Labels from device-resident channels-last ``(X, Y, Z, C)`` logits, or ``None`` if unsupported.

    Reference ``metal_restore.py:363-401``: ``None`` for a dtype other than
    float32/float16, a rank other than four, or a geometry/policy the kernel does
    not cover, so that the caller restores on the host.  Any strides are accepted
    (``predict_device_logits`` returns a channels-last view of channel-first logits).
    """
    if not isinstance(logits, torch.Tensor) or not logits.is_cuda or logits.dim() != 4:
        return None
    if logits.dtype not in (torch.float32, torch.float16):
        return None
    target = _target_shape(new_shape)
    classes = int(logits.shape[-1])
    source = tuple(int(v) for v in logits.shape[:3])
    if not device_class_restore_supported(source, target, current_spacing, new_spacing, contract, classes=classes):
        return None
    return kernels.to_host(restore_labels_on_device(logits, target, class_axis=3))


def _shape(value: object, *, name: str) -> tuple[int, int, int]:
    if not isinstance(value, list | tuple) or len(value) != 3 or any(
            isinstance(v, bool) or not isinstance(v, int | np.integer) or v < 1 for v in value):
        raise ContractError(f"{name} must contain three positive integers")
    return tuple(int(v) for v in value)  # type: ignore[return-value]


def _bounding_box(value: object, shape: tuple[int, int, int]) -> tuple[tuple[int, int], ...]:
    """``bbox_used_for_cropping`` as three half-open pairs inside ``shape`` (reference ``export.py:760-786``)."""
    if not isinstance(value, list | tuple) or len(value) != 3:
        raise ContractError("bbox_used_for_cropping must contain three pairs")
    result = []
    for axis, pair in enumerate(value):
        if not isinstance(pair, list | tuple) or len(pair) != 2:
            raise ContractError("bbox_used_for_cropping must contain three pairs")
        start, stop = pair
        if (any(isinstance(v, bool) or not isinstance(v, int | np.integer) for v in (start, stop))
                or not 0 <= start < stop <= shape[axis]):
            raise ContractError("bbox_used_for_cropping is outside the original shape")
        result.append((int(start), int(stop)))
    return tuple(result)


def _prediction_resampling_spacings(properties: Mapping[str, object], plans: PlansContract,
                                    crop_shape: tuple[int, int, int]):
    """Plans-grid and original-grid spacings, both in the plans' axis order (reference ``export.py:418-444``)."""
    spacing = properties.get("spacing")
    if not isinstance(spacing, list | tuple) or len(spacing) != 3:
        raise ContractError("prediction properties spacing must contain three values")
    spacing = validate_spacing(spacing, name="spacing")
    transposed = tuple(spacing[a] for a in plans.transpose_forward)
    configured = tuple(plans.configuration.spacing)
    if len(configured) != len(crop_shape):
        configured = (transposed[0], *configured)
    current = tuple(original if c is None else float(c) for c, original in zip(configured, transposed, strict=True))
    return current, transposed


def can_restore_device_segmentation(source_shape: Sequence[int], properties: Mapping[str, object],
                                    plans: PlansContract, semantics: LabelSemantics) -> bool:
    """Preflight of ``restore_device_segmentation`` before any logits exist (reference ``export.py:305-320``)."""
    if semantics.has_regions or len(source_shape) != 3:
        return False
    crop_shape = _shape(properties.get("shape_after_cropping_and_before_resampling"),
                        name="shape_after_cropping_and_before_resampling")
    current, original = _prediction_resampling_spacings(properties, plans, crop_shape)
    return device_class_restore_supported(source_shape, crop_shape, current, original,
                                          plans.configuration.probability_resampling,
                                          classes=semantics.output_channels)


def restore_device_segmentation(logits: torch.Tensor, properties: Mapping[str, object], plans: PlansContract,
                                semantics: LabelSemantics) -> RestoredPrediction | None:
    """Labels in the image's grid from device channels-last ``(*spatial, C)`` logits, or ``None``.

    Reference ``export.py:323-373``: resample to the crop, argmax, uncrop into
    ``shape_before_cropping`` at ``bbox_used_for_cropping`` and transpose by the
    plans' ``transpose_backward``.  Here all of it runs in one kernel and only the
    final uint16 volume is copied to the host.
    """
    if (semantics.has_regions or not isinstance(logits, torch.Tensor) or logits.dim() != 4
            or int(logits.shape[-1]) != semantics.output_channels):
        raise ContractError("device restoration requires class logits matching the output contract")
    shape_before = _shape(properties.get("shape_before_cropping"), name="shape_before_cropping")
    crop_shape = _shape(properties.get("shape_after_cropping_and_before_resampling"),
                        name="shape_after_cropping_and_before_resampling")
    box = _bounding_box(properties.get("bbox_used_for_cropping"), shape_before)
    current, original = _prediction_resampling_spacings(properties, plans, crop_shape)
    if not logits.is_cuda or logits.dtype not in (torch.float32, torch.float16):
        return None
    source = tuple(int(v) for v in logits.shape[:3])
    if not device_class_restore_supported(source, crop_shape, current, original,
                                          plans.configuration.probability_resampling,
                                          classes=semantics.output_channels):
        return None
    extents = tuple(stop - start for start, stop in box)
    if extents != crop_shape:
        raise ContractError(f"restored crop shape {crop_shape} does not match bbox {extents}")
    labels = restore_labels_on_device(logits, crop_shape, class_axis=3, volume_shape=shape_before,
                                      crop_lo=tuple(start for start, _ in box),
                                      axes=tuple(int(a) for a in plans.transpose_backward))
    return RestoredPrediction(segmentation=kernels.to_host(labels), probabilities=None)


def plans_from_payload(payload: Mapping[str, object], *, configuration: str) -> PlansContract:
    """The restoration view of a plans file: transposes, target spacing, probability resampling."""
    from nnunet_mlx_b200.data.preprocessing import ResamplingContract as PlanEntry

    forward = payload.get("transpose_forward")
    if not isinstance(forward, list | tuple) or sorted(forward) != [0, 1, 2]:
        raise ContractError("transpose_forward must be a permutation of [0, 1, 2]")
    forward = tuple(int(a) for a in forward)
    inverse = tuple(forward.index(a) for a in range(3))
    backward = tuple(int(a) for a in payload.get("transpose_backward", inverse))
    if backward != inverse:
        raise ContractError("transpose_backward is not the inverse of transpose_forward")
    configurations = payload.get("configurations")
    if not isinstance(configurations, Mapping) or not isinstance(configurations.get(configuration), Mapping):
        raise ContractError(f"plans have no configuration {configuration!r}")
    config = configurations[configuration]
    entry = PlanEntry.from_configuration(config, field="resampling_fn_probabilities", expected_is_seg=False)
    spacing = tuple(None if v is None else float(v) for v in config.get("spacing", ()))
    return PlansContract(forward, backward, ConfigurationContract(spacing, ResamplingContract(
        entry.function_name, entry.order, entry.order_z, entry.force_separate_z,
        entry.separate_z_anisotropy_threshold)))


def restore_segmentation_on_device(logits: torch.Tensor, properties: Mapping[str, object], plans: PlansContract,
                                   semantics: LabelSemantics, *, probability_resampling=None) -> RestoredPrediction:
    """Labels in the image's grid from device channels-last logits under every supported policy.

    Where the fused kernel applies this is ``restore_device_segmentation``.  Otherwise (spline plans
    with a separate axis or order 3, torch-grid plans) the float32 class logits are resampled to the
    crop grid on the device with the preprocessing kernels -- the arithmetic of the reference's host
    path (``resample_class_logits_argmax``, reference ``prediction/restore.py:73-103``: the probability
    contract's resampling of the logits, then the first argmax) -- and reduced, uncropped and
    transposed by the identity-grid kernel.  ``probability_resampling`` is the plan entry parsed with
    its torch-grid modes (``data.preprocessing.ResamplingContract``); without it the plans' spline
    entry is used.  Raises ``ContractError`` where no device path exists (region models, half logits
    off the fused path, spline orders other than 1 and 3).
    """
    fused = restore_device_segmentation(logits, properties, plans, semantics)
    if fused is not None:
        return fused
    from nnunet_mlx_b200.data import preprocessing as pre

    if logits.dtype != torch.float32:
        raise ContractError("device restoration off the fused kernel needs float32 logits")
    shape_before = _shape(properties.get("shape_before_cropping"), name="shape_before_cropping")
    crop_shape = _shape(properties.get("shape_after_cropping_and_before_resampling"),
                        name="shape_after_cropping_and_before_resampling")
    box = _bounding_box(properties.get("bbox_used_for_cropping"), shape_before)
    if tuple(stop - start for start, stop in box) != crop_shape:
        raise ContractError("restored crop shape does not match bbox_used_for_cropping")
    current, original = _prediction_resampling_spacings(properties, plans, crop_shape)
    contract = probability_resampling or plans.configuration.probability_resampling
    values = logits.permute(3, 0, 1, 2)  # classes first, a view
    if contract.function_name == "resample_torch_fornnunet":
        resampled = pre.resample_torch_device(values, crop_shape, current, original, contract, is_seg=False)
    else:
        resampled = pre.resample_spline_device(values, crop_shape, current, original, contract)
    labels = restore_labels_on_device(resampled, crop_shape, class_axis=0, volume_shape=shape_before,
                                      crop_lo=tuple(start for start, _ in box),
                                      axes=tuple(int(a) for a in plans.transpose_backward))
    return RestoredPrediction(segmentation=kernels.to_host(labels), probabilities=None)
