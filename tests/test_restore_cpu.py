"""Class-label restoration on the CPU: the oracle pinned to the reference, and the host-side policy.

The oracle (``oracle/restore.py``) is checked two ways: against scipy's order-1
``zoom`` (the arithmetic of the reference's host path, which the reference's own
device test compares labels with, ``tests/test_metal_restore.py:39-76``), value for
value; and against the per-axis grid of the reference's fused kernel, recorded
from its ``_axis_metadata`` in ``tests/golden/restore_axes.npz``.  The product's
support decisions are checked against ``tests/golden/restore_policy.json``,
recorded from the reference's ``device_class_restore_supported`` and
``separate_z_axis``.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch
from scipy import ndimage

from nnunet_mlx_b200 import kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.prediction import restore
from oracle import restore as orestore

GOLDEN = Path(__file__).resolve().parent / "golden"

# The reference's device-restoration parity shapes (classes, source, target).
REFERENCE_CASES = [
    (2, (2, 3, 4), (3, 5, 7)),
    (3, (5, 7, 11), (3, 4, 6)),
    (32, (1, 5, 7), (3, 7, 1)),
    (118, (4, 5, 6), (7, 8, 9)),
    (3, (2, 3, 5), (2, 3, 5)),
]


def _random_cases(count: int, seed: int):
    rng = np.random.default_rng(seed)
    for _ in range(count):
        yield (int(rng.integers(1, 6)), tuple(int(v) for v in rng.integers(1, 24, 3)),
               tuple(int(v) for v in rng.integers(1, 24, 3)))


def _host_path(logits: np.ndarray, target) -> np.ndarray:
    """The reference's host order-1 path: scipy zoom in float64, one cast to the input dtype."""
    if tuple(logits.shape[1:]) == tuple(target):
        return logits.astype(np.float32)
    source = logits if logits.dtype == np.float32 else logits.astype(np.float64)
    out = np.empty((logits.shape[0], *target), dtype=source.dtype)
    for c in range(logits.shape[0]):
        ndimage.zoom(source[c], np.divide(target, logits.shape[1:]), output=out[c], order=1, mode="nearest",
                     grid_mode=True)
    return out.astype(logits.dtype)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("classes,source,target", REFERENCE_CASES + list(_random_cases(24, 5)))
def test_oracle_values_equal_the_host_spline_path(classes, source, target, dtype):
    """Values equal scipy's bit for bit; labels equal its first argmax (half logits: frequent ties)."""
    scale = 0.01 if dtype is np.float16 else 1.0
    logits = np.random.default_rng(classes).normal(scale=scale, size=(classes, *source)).astype(dtype)
    expected = _host_path(logits, target)
    values = orestore.rounded_values(logits, target)
    np.testing.assert_array_equal(values.astype(np.float32), expected.astype(np.float32))
    labels = orestore.restore_labels(logits, target)
    np.testing.assert_array_equal(labels, np.argmax(expected, axis=0).astype(np.uint16))


def test_oracle_grid_matches_the_reference_axis_metadata():
    """Per target index, the weight each source voxel receives equals the reference kernel's grid."""
    golden = np.load(GOLDEN / "restore_axes.npz")
    pairs = sorted({tuple(int(v) for v in k.split("_")[:2]) for k in golden.files})
    assert len(pairs) >= 20
    for source, target in pairs:
        key = f"{source}_{target}_"
        ref = np.zeros((target, source))
        rows = np.arange(target)
        np.add.at(ref, (rows, golden[key + "lower"]),
                  golden[key + "lower_high"].astype(np.float64) + golden[key + "lower_low"])
        np.add.at(ref, (rows, golden[key + "upper"]),
                  golden[key + "upper_high"].astype(np.float64) + golden[key + "upper_low"])
        i0, i1, w0, w1 = orestore.axis_taps(source, target)
        mine = np.zeros((target, source))
        np.add.at(mine, (rows, i0), w0)
        np.add.at(mine, (rows, i1), w1)
        np.testing.assert_allclose(mine, ref, rtol=0, atol=1e-13, err_msg=f"{source} -> {target}")


def test_oracle_uncrop_and_transpose():
    logits = np.random.default_rng(3).normal(size=(4, 5, 6, 7)).astype(np.float32)
    labels = orestore.restore_labels(logits, (6, 4, 9), volume=(9, 8, 12), crop_lo=(2, 1, 3), axes=(2, 0, 1))
    inner = orestore.first_argmax(orestore.rounded_values(logits, (6, 4, 9)))
    full = np.zeros((9, 8, 12), np.uint16)
    full[2:8, 1:5, 3:12] = inner
    np.testing.assert_array_equal(labels, full.transpose(2, 0, 1))


def _contract(entry) -> restore.ResamplingContract:
    fn, order, order_z, force, threshold = entry
    return restore.ResamplingContract(fn, order, order_z, force, separate_z_anisotropy_threshold=threshold)


def test_support_decisions_match_the_reference():
    policy = json.loads((GOLDEN / "restore_policy.json").read_text())
    for case in policy["support"]:
        got = restore.device_class_restore_supported(case["source"], case["target"], case["current"], case["new"],
                                                     _contract(case["contract"]), classes=case["classes"])
        assert got == case["supported"], case
    for case in policy["separate_z"]:
        got = restore.separate_z_axis(tuple(case["current"]), tuple(case["new"]), force=case["force"],
                                      threshold=case["threshold"])
        assert got == (case["separate"], case["axis"]), case


def _plans(transpose_forward=(0, 1, 2), spacing=(1.0, 1.0, 1.0), order=1):
    backward = tuple(int(i) for i in np.argsort(transpose_forward))
    contract = restore.ResamplingContract("resample_data_or_seg_to_shape", order, 0, None)
    return restore.PlansContract(tuple(transpose_forward), backward,
                                 restore.ConfigurationContract(tuple(spacing), contract))


def test_preflight_resolves_spacings_in_plans_axis_order():
    props = {"spacing": [0.9, 0.9, 2.5], "shape_after_cropping_and_before_resampling": [40, 50, 60],
             "shape_before_cropping": [45, 60, 70], "bbox_used_for_cropping": [[0, 40], [5, 55], [3, 63]]}
    plans = _plans((2, 0, 1), spacing=(2.5, 1.0, 1.0))
    current, original = restore._prediction_resampling_spacings(props, plans, (40, 50, 60))
    assert original == (2.5, 0.9, 0.9) and current == (2.5, 1.0, 1.0)
    sem = restore.LabelSemantics(3)
    assert restore.can_restore_device_segmentation((40, 40, 48), props, plans, sem)
    assert not restore.can_restore_device_segmentation((40, 40, 48), props, _plans((2, 0, 1), (2.5, 1, 1), 3), sem)
    assert restore.can_restore_device_segmentation((40, 50, 60), props, _plans((2, 0, 1), (2.5, 1, 1), 3), sem)
    assert not restore.can_restore_device_segmentation((40, 40, 48), props, plans, restore.LabelSemantics(3, True))
    anisotropic = dict(props, spacing=[0.8, 0.8, 2.5])  # 2.5 / 0.8 > 3: separate-axis resampling
    assert not restore.can_restore_device_segmentation((40, 40, 48), anisotropic, plans, sem)
    two_d = restore.PlansContract((2, 0, 1), (1, 2, 0), restore.ConfigurationContract(
        (1.0, 1.0), restore.ResamplingContract("resample_data_or_seg_to_shape", 1, 0, None)))
    assert restore._prediction_resampling_spacings(props, two_d, (40, 50, 60))[0] == (2.5, 1.0, 1.0)


@pytest.mark.parametrize("bad", [
    {"bbox_used_for_cropping": [[0, 40], [5, 55]]},
    {"bbox_used_for_cropping": [[0, 46], [5, 55], [3, 63]]},
    {"bbox_used_for_cropping": [[3, 3], [5, 55], [3, 63]]},
    {"shape_before_cropping": [45, 60]},
    {"spacing": [0.8, -1.0, 2.5]},
])
def test_restore_device_segmentation_rejects_bad_properties(bad):
    props = {"spacing": [0.8, 0.8, 2.5], "shape_after_cropping_and_before_resampling": [40, 50, 60],
             "shape_before_cropping": [45, 60, 70], "bbox_used_for_cropping": [[0, 40], [5, 55], [3, 63]]}
    props.update(bad)
    logits = torch.zeros((40, 50, 60, 3))
    with pytest.raises(ContractError):
        restore.restore_device_segmentation(logits, props, _plans(), restore.LabelSemantics(3))


def test_restore_device_segmentation_contract_checks_before_the_device():
    props = {"spacing": [1.0, 1.0, 1.0], "shape_after_cropping_and_before_resampling": [4, 5, 6],
             "shape_before_cropping": [4, 5, 6], "bbox_used_for_cropping": [[0, 4], [0, 5], [0, 6]]}
    with pytest.raises(ContractError):  # channel count differs from the label semantics
        restore.restore_device_segmentation(torch.zeros((4, 5, 6, 2)), props, _plans(), restore.LabelSemantics(3))
    with pytest.raises(ContractError):  # regions are not class logits
        restore.restore_device_segmentation(torch.zeros((4, 5, 6, 3)), props, _plans(),
                                            restore.LabelSemantics(3, True))
    # host tensors are not device logits: the caller restores on the host
    assert restore.restore_device_segmentation(torch.zeros((4, 5, 6, 3)), props, _plans(),
                                               restore.LabelSemantics(3)) is None
    assert restore.resample_device_logits_argmax(torch.zeros((4, 5, 6, 3)), (4, 5, 6), (1, 1, 1), (1, 1, 1),
                                                 _plans().configuration.probability_resampling) is None


@pytest.mark.parametrize("logits", [
    np.zeros((3, 4, 5), np.float32),
    np.zeros((0, 4, 5, 6), np.float32),
    np.zeros((3, 4, 5, 6), np.float64),
    np.full((3, 4, 5, 6), np.inf, np.float32),
])
def test_host_entry_rejects_bad_logits_before_the_device(logits):
    with pytest.raises(ContractError):
        restore.resample_class_logits_argmax_device(logits, (4, 5, 6))


def test_kernel_wrapper_refuses_host_tensors():
    with pytest.raises(ContractError):
        kernels.restore_class_labels(torch.zeros((3, 4, 5, 6)), (4, 5, 6))
