"""Array predictor (fold ensemble) and host probability/label helpers.

Drop-in for reference ``src/nnunet_mlx/prediction/inference.py``:
``average_fold_logits`` (25-90), ``average_fold_device_logits`` (93-149),
``logits_to_probabilities`` (210-233), ``probabilities_to_segmentation``
(246-269) and ``ArrayPredictor`` (280-339) -- the seam
``ModelFolderPredictor`` constructs (reference ``prediction/pipeline.py:207-215``).
Models are this package's B200 networks; all folds run inside one device
sliding window (``prediction.sliding_window.predict_volume``).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction.sliding_window import _check_accumulation, predict_volume


def average_fold_logits(models, data_channels_first, *, patch_size, num_outputs: int, mirroring_axes=(),
                        step_fraction: float = 0.5, accumulation: str = "float32") -> np.ndarray:
    """Host ``(num_outputs, *spatial)`` fold-averaged logits: float32, or float16 for ``nnunet-fp16``
    (each fold rounded to float16, summed in order and divided, as upstream keeps half tensors)."""
    _check_accumulation(accumulation)
    if not models:
        raise ContractError("fold inference requires at least one model")
    half = accumulation == "nnunet-fp16"
    logits, _ = predict_volume(list(models), data_channels_first, patch_size=patch_size, num_classes=num_outputs,
                               mirroring_axes=mirroring_axes, step_fraction=step_fraction, label_dtype=None,
                               accumulation=accumulation, half_logits=half)
    return kernels.to_host(logits)


def average_fold_device_logits(models, data_channels_first, *, patch_size, num_outputs: int, mirroring_axes=(),
                               step_fraction: float = 0.5, accumulation: str = "float32") -> torch.Tensor:
    """Device fold-averaged logits, channels-last ``(*spatial, C)`` (a view of the channel-first result);
    float16 for ``nnunet-fp16``."""
    _check_accumulation(accumulation)
    if not models:
        raise ContractError("fold inference requires at least one model")
    logits, _ = predict_volume(list(models), data_channels_first, patch_size=patch_size, num_classes=num_outputs,
                               mirroring_axes=mirroring_axes, step_fraction=step_fraction, label_dtype=None,
                               accumulation=accumulation, half_logits=True)
    return logits.permute(1, 2, 3, 0)


def logits_to_probabilities(logits, *, has_regions: bool) -> np.ndarray:
    """Softmax over channels (classes) or independent sigmoids (regions), float32."""
    values = np.asarray(logits, dtype=np.float32)
    if values.ndim not in (3, 4) or not np.isfinite(values).all():
        raise ContractError(f"expected finite channel-first 2-D/3-D logits, got {values.shape}")
    if has_regions:
        out = np.empty_like(values)
        pos = values >= 0
        out[pos] = 1 / (1 + np.exp(-values[pos]))
        e = np.exp(values[~pos])
        out[~pos] = e / (1 + e)
        return out
    shifted = values - values.max(axis=0, keepdims=True)
    np.exp(shifted, out=shifted)
    shifted /= shifted.sum(axis=0, keepdims=True)
    return np.ascontiguousarray(shifted, dtype=np.float32)


def probabilities_to_segmentation(probabilities, *, regions_class_order: Sequence[int] | None) -> np.ndarray:
    """uint16 labels: argmax for classes, later-channel-wins thresholding at 0.5 for regions."""
    values = np.asarray(probabilities, dtype=np.float32)
    if values.ndim not in (3, 4) or not np.isfinite(values).all():
        raise ContractError(f"expected finite channel-first 2-D/3-D probabilities, got {values.shape}")
    if regions_class_order is None:
        return np.asarray(np.argmax(values, axis=0), dtype=np.uint16)
    order = tuple(int(v) for v in regions_class_order)
    if len(order) != values.shape[0] or any(v < 1 for v in order):
        raise ContractError("regions_class_order does not match output channels")
    seg = np.zeros(values.shape[1:], dtype=np.uint16)
    for channel, label in enumerate(order):
        seg[values[channel] > 0.5] = label
    return seg


class ArrayPredictor:
    """Predict from preprocessed ``(C, *spatial)`` arrays with a fold ensemble on one B200."""

    def __init__(self, models, *, patch_size, num_outputs: int, mirroring_axes: Sequence[int] = (),
                 regions_class_order: Sequence[int] | None = None, step_fraction: float = 0.5,
                 accumulation: str = "float32") -> None:
        if regions_class_order is None and num_outputs < 2:
            raise ContractError("class inference requires at least two output channels")
        if not models:
            raise ContractError("predictor requires at least one fold model")
        _check_accumulation(accumulation)
        for model in models:
            if not hasattr(model, "forward_features"):
                raise ContractError("fold models must be B200 networks (nnunet_mlx_b200.model.network)")
        self.models = tuple(models)
        self.patch_size = tuple(int(v) for v in patch_size)
        self.num_outputs = num_outputs
        self.mirroring_axes = tuple(int(a) for a in mirroring_axes)
        self.regions_class_order = None if regions_class_order is None else tuple(regions_class_order)
        self.step_fraction = step_fraction
        self.accumulation = accumulation

    def predict_logits_from_preprocessed_data(self, data_channels_first) -> np.ndarray:
        """Fold-averaged host float32 logits ``(num_outputs, *spatial)``."""
        return average_fold_logits(self.models, data_channels_first, patch_size=self.patch_size,
                                   num_outputs=self.num_outputs, mirroring_axes=self.mirroring_axes,
                                   step_fraction=self.step_fraction, accumulation=self.accumulation)

    def predict_device_logits_from_preprocessed_data(self, data_channels_first) -> torch.Tensor:
        """Fold-averaged device logits, channels-last ``(*spatial, C)``."""
        return average_fold_device_logits(self.models, data_channels_first, patch_size=self.patch_size,
                                          num_outputs=self.num_outputs, mirroring_axes=self.mirroring_axes,
                                          step_fraction=self.step_fraction, accumulation=self.accumulation)

    def predict_labels_from_preprocessed_data(self, data_channels_first) -> np.ndarray:
        """Class labels computed on the device; only labels are copied to the host."""
        if self.regions_class_order is not None:
            raise ContractError("device labels are defined for class (softmax) models")
        _, labels = predict_volume(list(self.models), data_channels_first, patch_size=self.patch_size,
                                   num_classes=self.num_outputs, mirroring_axes=self.mirroring_axes,
                                   step_fraction=self.step_fraction, want_logits=False,
                                   label_dtype=torch.uint8 if self.num_outputs <= 255 else torch.uint16,
                                   accumulation=self.accumulation)
        return kernels.to_host(labels).astype(np.uint16)
