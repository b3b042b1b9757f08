"""Class-label restoration on B200 (``nnb_restore_class_labels``) against the oracle.

Labels are index work: they must equal the oracle's exactly, including the
frequent near-ties of small half logits (``oracle/restore.py`` equals the
reference's host spline path value for value; ``tests/test_restore_cpu.py``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction import restore
from oracle import restore as orestore

pytestmark = pytest.mark.gpu

CASES = [
    (2, (2, 3, 4), (3, 5, 7)),
    (3, (5, 7, 11), (3, 4, 6)),
    (32, (1, 5, 7), (3, 7, 1)),
    (118, (4, 5, 6), (7, 8, 9)),
    (3, (2, 3, 5), (2, 3, 5)),
    (1, (4, 4, 4), (9, 3, 5)),
    (3, (1, 1, 1), (2, 3, 4)),
    (5, (33, 17, 40), (21, 35, 40)),
    (300, (3, 4, 5), (5, 4, 3)),
    (6, (7, 9, 70), (7, 9, 70)),
    (4, (3, 5, 300), (3, 5, 300)),
]


def _logits(classes, source, dtype, seed):
    scale = 0.01 if dtype is np.float16 else 1.0
    return np.random.default_rng(seed).normal(scale=scale, size=(classes, *source)).astype(dtype)


def _device(values: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(values).to(device)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("classes,source,target", CASES)
def test_labels_equal_the_oracle(cuda_device, classes, source, target, dtype):
    values = _logits(classes, source, dtype, classes)
    labels = restore.restore_labels_on_device(_device(values, cuda_device), target, class_axis=0)
    np.testing.assert_array_equal(kernels.to_host(labels), orestore.restore_labels(values, target))


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_channels_last_layouts_and_views(cuda_device, dtype):
    values = _logits(4, (9, 10, 11), dtype, 11)
    expected = orestore.restore_labels(values, (13, 7, 15))
    channel_first = _device(values, cuda_device)
    view = channel_first.permute(1, 2, 3, 0)                 # what predict_device_logits returns
    contiguous = view.contiguous()
    for logits in (view, contiguous):
        labels = restore.restore_labels_on_device(logits, (13, 7, 15), class_axis=3)
        np.testing.assert_array_equal(kernels.to_host(labels), expected)
    sliced = _device(_logits(4, (12, 10, 11), dtype, 12), cuda_device)[:, 2:11]
    np.testing.assert_array_equal(
        kernels.to_host(restore.restore_labels_on_device(sliced, (13, 7, 15), class_axis=0)),
        orestore.restore_labels(sliced.cpu().numpy(), (13, 7, 15)))


@pytest.mark.parametrize("axes", [(0, 1, 2), (2, 0, 1), (1, 2, 0), (2, 1, 0)])
@pytest.mark.parametrize("label_dtype", [torch.uint16, torch.uint8])
def test_uncrop_and_axis_order(cuda_device, axes, label_dtype):
    values = _logits(3, (6, 8, 10), np.float32, 5)
    target, volume, lo = (7, 9, 12), (10, 11, 20), (1, 0, 6)
    labels = restore.restore_labels_on_device(_device(values, cuda_device), target, class_axis=0, volume_shape=volume,
                                              crop_lo=lo, axes=axes, label_dtype=label_dtype)
    assert labels.dtype == label_dtype and tuple(labels.shape) == tuple(volume[a] for a in axes)
    expected = orestore.restore_labels(values, target, volume=volume, crop_lo=lo, axes=axes)
    np.testing.assert_array_equal(kernels.to_host(labels).astype(np.uint16), expected)


@pytest.mark.parametrize("axes", [(0, 1, 2), (2, 0, 1), (1, 2, 0), (2, 1, 0)])
@pytest.mark.parametrize("classes", [3, 7])
def test_identity_grid_uncrop_and_axis_order(cuda_device, axes, classes):
    """Equal grids take the argmax-only kernel; the uncrop and axis order are the same."""
    values = _logits(classes, (7, 9, 300), np.float16, classes)
    volume, lo = (10, 11, 310), (3, 1, 7)
    labels = restore.restore_labels_on_device(_device(values, cuda_device), (7, 9, 300), class_axis=0,
                                              volume_shape=volume, crop_lo=lo, axes=axes)
    expected = orestore.restore_labels(values, (7, 9, 300), volume=volume, crop_lo=lo, axes=axes)
    np.testing.assert_array_equal(kernels.to_host(labels), expected)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("view", ["full", "tail", "short", "shifted"])
@pytest.mark.parametrize("classes", [3, 6])
def test_identity_rows_vector_and_scalar_reads(cuda_device, dtype, view, classes):
    """Aligned contiguous rows take 4-element vector reads (with a scalar tail); a shifted view does not."""
    whole = _device(_logits(classes, (7, 9, 300), dtype, classes + 1), cuda_device)
    logits = {"full": whole, "tail": whole[..., :298], "short": whole[..., :5], "shifted": whole[..., 2:300]}[view]
    target = tuple(int(v) for v in logits.shape[1:])
    volume, lo = (target[0] + 3, target[1] + 2, target[2] + 9), (1, 2, 3)
    for axes in [(0, 1, 2), (1, 0, 2), (2, 0, 1)]:
        labels = restore.restore_labels_on_device(logits, target, class_axis=0, volume_shape=volume, crop_lo=lo,
                                                  axes=axes)
        expected = orestore.restore_labels(logits.cpu().numpy(), target, volume=volume, crop_lo=lo, axes=axes)
        np.testing.assert_array_equal(kernels.to_host(labels), expected)


def _plans(transpose_forward, spacing, order=1):
    backward = tuple(int(i) for i in np.argsort(transpose_forward))
    contract = restore.ResamplingContract("resample_data_or_seg_to_shape", order, 0, None)
    return restore.PlansContract(tuple(transpose_forward), backward,
                                 restore.ConfigurationContract(tuple(spacing), contract))


def test_restore_device_segmentation_matches_the_export_path(cuda_device):
    """Resample + argmax + uncrop + transpose_backward in one call equals the oracle's export steps."""
    props = {"spacing": [0.9, 0.9, 2.5], "shape_after_cropping_and_before_resampling": [20, 30, 36],
             "shape_before_cropping": [24, 40, 44], "bbox_used_for_cropping": [[2, 22], [5, 35], [4, 40]]}
    plans = _plans((2, 0, 1), (2.5, 1.2, 1.2))
    values = _logits(3, (20, 22, 27), np.float32, 9)                  # network-grid logits, (C, *spatial)
    logits = _device(values, cuda_device).permute(1, 2, 3, 0)      # device channels-last view
    sem = restore.LabelSemantics(3)
    assert restore.can_restore_device_segmentation(tuple(logits.shape[:3]), props, plans, sem)
    restored = restore.restore_device_segmentation(logits, props, plans, sem)
    assert restored is not None and restored.probabilities is None
    expected = orestore.restore_labels(values, (20, 30, 36), volume=(24, 40, 44), crop_lo=(2, 5, 4),
                                       axes=plans.transpose_backward)
    assert restored.segmentation.dtype == np.uint16
    np.testing.assert_array_equal(restored.segmentation, expected)
    # an order-3 plan is not the device kernel's: the caller restores on the host
    assert restore.restore_device_segmentation(logits, props, _plans((2, 0, 1), (2.5, 1.2, 1.2), 3), sem) is None


def test_host_and_device_entry_points(cuda_device):
    values = _logits(118, (4, 5, 6), np.float16, 118)
    expected = orestore.restore_labels(values, (7, 8, 9))
    np.testing.assert_array_equal(restore.resample_class_logits_argmax_device(values, (7, 8, 9)), expected)
    logits = _device(values, cuda_device).permute(1, 2, 3, 0)
    order1 = restore.ResamplingContract("resample_data_or_seg_to_shape", 1, 0, False)
    order3 = restore.ResamplingContract("resample_data_or_seg_to_shape", 3, 0, False)
    np.testing.assert_array_equal(restore.resample_device_logits_argmax(logits, (7, 8, 9), (1, 1, 1), (1, 1, 1),
                                                                        order1), expected)
    assert restore.resample_device_logits_argmax(logits, (7, 8, 9), (1, 1, 1), (1, 1, 1), order3) is None
    same = restore.resample_device_logits_argmax(logits, (4, 5, 6), (1, 1, 1), (1, 1, 1), order3)
    np.testing.assert_array_equal(same, orestore.restore_labels(values, (4, 5, 6)))


def test_non_finite_values_raise(cuda_device):
    values = _logits(3, (5, 6, 7), np.float32, 1)
    values[1, 2, 3, 4] = np.inf
    logits = _device(values, cuda_device)
    with pytest.raises(ContractError):
        restore.restore_labels_on_device(logits, (8, 8, 8), class_axis=0)
    labels, invalid = kernels.restore_class_labels(logits, (8, 8, 8))
    count = int(invalid.item())
    assert count > 0 and int((kernels.to_host(labels) == 0xFFFF).sum()) == count


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_larger_grids(cuda_device, dtype):
    """A few million target voxels: up-sampled in-plane, down-sampled along axis 0, and an identity slab."""
    values = _logits(3, (48, 150, 170), dtype, 48)
    target = (40, 256, 300)
    labels = restore.restore_labels_on_device(_device(values, cuda_device), target, class_axis=0)
    np.testing.assert_array_equal(kernels.to_host(labels), orestore.restore_labels(values, target))
    slab = _logits(3, (8, 768, 768), dtype, 8)
    labels = restore.restore_labels_on_device(_device(slab, cuda_device), (8, 768, 768), class_axis=0)
    np.testing.assert_array_equal(kernels.to_host(labels), orestore.first_argmax(slab))



def test_zero_weight_corner_is_not_read(cuda_device):
    """A corner of interpolation weight exactly 0 is skipped, so a non-finite value there is not seen.

    Only z is resampled (y and x keep their size: every upper weight there is
    exactly 0).  The inf at x = 5 is the zero-weight upper x corner of the
    voxels at x = 4, which keep the label of the finite data and are not
    counted invalid (the host sum would give NaN there); the voxels at x = 5
    read it with a nonzero weight and are counted.  The contract is finite
    logits, which the host entry point checks before the launch.
    """
    values = _logits(3, (4, 5, 6), np.float32, 21)
    finite = values.copy()
    values[1, 2, 3, 5] = np.inf
    target = (7, 5, 6)
    labels, invalid = kernels.restore_class_labels(_device(values, cuda_device), target, class_axis=0)
    got = kernels.to_host(labels).astype(np.uint16)
    expected = orestore.restore_labels(finite, target)
    mask = np.ones(target, dtype=bool)
    mask[:, 3, 5] = False
    np.testing.assert_array_equal(got[mask], expected[mask])
    hit = int((got[:, 3, 5] == 65535).sum())
    assert hit > 0 and int(invalid.item()) == hit
    with pytest.raises(ContractError):
        restore.resample_class_logits_argmax_device(values, target)
