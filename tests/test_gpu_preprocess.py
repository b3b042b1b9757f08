"""Device raw-case preprocessing against upstream's recorded vectors and the CPU oracle (needs a B200).

Everything runs through the C ABI (``nnb_nonzero_bounds``, ``nnb_fill_holes_*``,
``nnb_crop_labels``, ``nnb_crop_normalize``, ``nnb_torch_resize``).  Bars: labels, bounding
boxes and crop shapes exactly; image values bitwise equal to the oracle where the arithmetic
has no reduction (crop, CT / rescale / RGB normalisation, torch-grid interpolation), and within
the reference's own preprocessing tolerance (rtol 1e-5, atol 5e-6,
``tests/test_torch_resampling.py:84-86``) where a z-score mean and standard deviation are reduced
(float64 sums on the device, NumPy's float32 pairwise sums in the oracle) and for spline
resampling against scipy ``zoom`` (float64 on both sides, one rounding to float32).
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import preprocess as op

from .conftest import GOLDEN

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6
SCHEMES = ("CTNormalization", "ZScoreNormalization", "NoNormalization", "RescaleTo01Normalization",
           "RGBTo01Normalization")
DTYPES = (np.float32, np.float64, np.int16, np.uint8, np.uint16, np.int32)


def _recorded():
    saved = np.load(GOLDEN / "torch_resampling_labels.npz")
    return saved, json.loads(str(saved["metadata"].item()))


def _contract(kwargs):
    from nnunet_mlx_b200.data.preprocessing import ResamplingContract

    return ResamplingContract("resample_torch_fornnunet", 1, 0, kwargs.get("force_separate_z"),
                              kwargs.get("seg_tiebreak", "nearest"), kwargs.get("mode", "linear"),
                              kwargs.get("aniso_axis_mode", "nearest-exact"),
                              kwargs.get("separate_z_anisotropy_threshold", 3.0))


def _status_clean():
    from nnunet_mlx_b200 import _native

    torch.cuda.synchronize()
    status, where = _native.device_status(reset=True)
    assert status == 0, f"device status {status} at {where}"


def test_device_label_resampling_matches_upstream_recording(cuda_device):
    from nnunet_mlx_b200.data.preprocessing import resample_torch_device

    saved, meta = _recorded()
    for case in meta["cases"]:
        source = torch.from_numpy(saved[f"{case['name']}-input"].astype(np.int32)).to(cuda_device)
        got = resample_torch_device(source, case["shape"], case["spacing"], case["new_spacing"],
                                    _contract(case["kwargs"]), is_seg=True).cpu().numpy()
        expected = saved[f"{case['name']}-expected"]
        assert got.shape == expected.shape, case["name"]
        np.testing.assert_array_equal(got, expected.astype(np.int64), err_msg=case["name"])
    _status_clean()


def test_device_preprocessing_matches_recorded_runs(cuda_device):
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case

    saved, meta = _recorded()
    for run in meta["pipeline"]:
        plans = PreprocessingPlans.from_payload(run["plans"], configuration="selected")
        result = preprocess_raw_case(saved["raw_nonzero"].astype(np.float32), run["properties"], plans,
                                     segmentation_previous_stage=saved["previous"], device=cuda_device)
        geometry = run["geometry"]
        assert list(result.properties["shape_before_cropping"]) == geometry["shape_before_cropping"]
        assert result.properties["bbox_used_for_cropping"] == geometry["bbox_used_for_cropping"]
        assert (list(result.properties["shape_after_cropping_and_before_resampling"])
                == geometry["shape_after_cropping_and_before_resampling"])
        np.testing.assert_array_equal(result.previous_stage.cpu().numpy(),
                                      saved[f"{run['name']}-labels"].astype(np.int64), err_msg=run["name"])
        assert result.data.is_cuda and result.data.dtype == torch.float32 and result.data.is_contiguous()
    _status_clean()


@pytest.mark.parametrize("seed", range(3))
def test_device_torch_resize_matches_oracle_bitwise(cuda_device, seed):
    from nnunet_mlx_b200 import kernels

    rng = np.random.default_rng(seed)
    for _ in range(12):
        source = tuple(int(v) for v in rng.integers(1, 24, 3))
        target = tuple(int(v) for v in rng.integers(1, 40, 3))
        values = (rng.standard_normal((2, *source)) * 10.0 ** rng.integers(-30, 30)).astype(np.float32)
        strided = torch.from_numpy(values).to(cuda_device).permute(0, 2, 1, 3)  # a view: strides, no copy
        host = np.ascontiguousarray(strided.cpu().numpy())
        for mode in ("linear", "nearest", "nearest-exact"):
            got = kernels.torch_resize(strided, target, mode).cpu().numpy()
            np.testing.assert_array_equal(got, op.torch_resize(host, target, mode, is_seg=False),
                                          err_msg=f"{mode} {source} -> {target}")
        labels = rng.integers(-1, 5, (1, *source)).astype(np.int32)
        for tiebreak in ("lowest", "highest", "nearest"):
            got = kernels.torch_resize(torch.from_numpy(labels).to(cuda_device), target, "linear", labels=True,
                                       tiebreak=tiebreak).cpu().numpy()
            np.testing.assert_array_equal(got, op.torch_resize(labels, target, "linear", is_seg=True,
                                                               tiebreak=tiebreak))
    _status_clean()


def _synthetic_case(rng, shape, dtype):
    """Nonzero block with an enclosed hole and a zero margin (so the crop is a strict sub-box)."""
    values = np.zeros(shape, dtype=np.float64)
    _, a, b, d = shape
    values[:, 1:a - 1, 2:b - 1, 1:d - 2] = rng.normal(50, 20, (shape[0], a - 2, b - 3, d - 3))
    values[:, a // 2, b // 2, d // 2] = 0
    values[0, 1, 2, 1] = 0
    if np.dtype(dtype).kind in "iu":
        values = np.clip(np.round(values), 0 if np.dtype(dtype).kind == "u" else -1000, 250)
    return values.astype(dtype)


def _plans(transpose, spacing, schemes, use_mask, intensity, data_kwargs, tiebreak):
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans

    payload = {"transpose_forward": list(transpose), "foreground_intensity_properties_per_channel": intensity,
               "configurations": {"c": {
                   "spacing": list(spacing), "normalization_schemes": list(schemes),
                   "use_mask_for_norm": list(use_mask), "resampling_fn_data": "resample_torch_fornnunet",
                   "resampling_fn_data_kwargs": data_kwargs, "resampling_fn_seg": "resample_torch_fornnunet",
                   "resampling_fn_seg_kwargs": {"is_seg": True, "seg_tiebreak": tiebreak}}}}
    return PreprocessingPlans.from_payload(payload, configuration="c")


@pytest.mark.parametrize("seed", range(4))
def test_device_preprocessing_matches_oracle(cuda_device, seed):
    from nnunet_mlx_b200.data.preprocessing import preprocess_raw_case

    rng = np.random.default_rng(100 + seed)
    for trial in range(12):
        channels = int(rng.integers(1, 4))
        schemes = [SCHEMES[int(rng.integers(0, 5))] for _ in range(channels)]
        use_mask = [bool(rng.integers(0, 2)) for _ in range(channels)]
        transpose = [int(v) for v in rng.permutation(3)]
        shape = (channels, *(int(v) for v in rng.integers(5, 20, 3)))
        dtype = DTYPES[(trial + seed) % len(DTYPES)]
        values = _synthetic_case(rng, shape, dtype)
        if "RGBTo01Normalization" in schemes:
            values = np.clip(values, 0, 255).astype(dtype)
        intensity = {str(c): {"mean": 40.5, "std": 17.25, "percentile_00_5": 10.0, "percentile_99_5": 90.0}
                     for c in range(channels)}
        spacing = [float(v) for v in rng.choice([0.7, 1.0, 1.6, 3.0, 5.0], 3)]
        target = [float(v) for v in rng.choice([0.8, 1.0, 1.4, 2.5], 3)]
        previous = rng.integers(0, 3, (1, *shape[1:])) if trial % 3 == 0 else None
        mode, aniso = (("linear", "nearest-exact"), ("nearest", "linear"), ("nearest-exact", "nearest"))[trial % 3]
        data_kwargs = {"is_seg": False, "mode": mode, "aniso_axis_mode": aniso}
        tiebreak = ("nearest", "lowest", "highest")[trial % 3]
        plans = _plans(transpose, target, schemes, use_mask, intensity, data_kwargs, tiebreak)
        result = preprocess_raw_case(values, {"spacing": spacing}, plans, segmentation_previous_stage=previous,
                                     device=cuda_device)
        reference, reference_previous, properties = op.preprocess(
            values, spacing, transpose_forward=transpose, configured_spacing=target, schemes=schemes,
            use_mask=use_mask, intensities=intensity,
            data_resampling=dict(mode=data_kwargs["mode"], aniso_axis_mode=data_kwargs["aniso_axis_mode"],
                                 force_separate_z=None, threshold=3.0),
            seg_resampling=dict(mode="linear", aniso_axis_mode="nearest-exact", force_separate_z=None,
                                threshold=3.0, tiebreak=tiebreak),
            previous=previous)
        assert result.properties["bbox_used_for_cropping"] == properties["bbox_used_for_cropping"]
        got = result.data.cpu().numpy()
        assert got.shape == reference.shape
        if "ZScoreNormalization" in schemes:
            np.testing.assert_allclose(got, reference, rtol=RTOL, atol=ATOL)
        else:
            np.testing.assert_array_equal(got, reference)
        if previous is not None:
            np.testing.assert_array_equal(result.previous_stage.cpu().numpy(), reference_previous.astype(np.int64))
    _status_clean()


def test_device_ct_volume_with_anisotropic_spacing(cuda_device):
    """A CT-like int16 volume: air -1000, zero margin, CT normalisation, in-plane 0.8 -> 1.0 mm."""
    from nnunet_mlx_b200.data.preprocessing import preprocess_raw_case

    rng = np.random.default_rng(7)
    raw = np.zeros((1, 40, 150, 150), dtype=np.int16)
    body = rng.normal(40, 15, (36, 140, 140)).clip(-1000, 3000)
    body[:, :20, :] = -1000
    raw[0, 2:38, 5:145, 4:144] = np.round(body).astype(np.int16)
    intensity = {"0": {"mean": 100.0, "std": 50.0, "percentile_00_5": -1000.0, "percentile_99_5": 400.0}}
    plans = _plans((0, 1, 2), (5.0, 1.0, 1.0), ["CTNormalization"], [False], intensity,
                   {"is_seg": False}, "nearest")
    result = preprocess_raw_case(raw, {"spacing": [5.0, 0.8, 0.8]}, plans, device=cuda_device)
    reference, _, properties = op.preprocess(
        raw, [5.0, 0.8, 0.8], transpose_forward=(0, 1, 2), configured_spacing=(5.0, 1.0, 1.0),
        schemes=["CTNormalization"], use_mask=[False], intensities=intensity,
        data_resampling=dict(mode="linear", aniso_axis_mode="nearest-exact", force_separate_z=None, threshold=3.0),
        seg_resampling=dict(mode="linear", aniso_axis_mode="nearest-exact", force_separate_z=None, threshold=3.0,
                            tiebreak="nearest"))
    assert result.properties["bbox_used_for_cropping"] == [[2, 38], [5, 145], [4, 144]]
    assert tuple(result.data.shape) == reference.shape == (1, 36, 112, 112)
    np.testing.assert_array_equal(result.data.cpu().numpy(), reference)
    _status_clean()


def test_device_preprocessing_feeds_the_predictor(cuda_device):
    """The preprocessed device tensor goes straight into the sliding window (no host round trip)."""
    from nnunet_mlx_b200.data.preprocessing import preprocess_raw_case
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume
    from nnunet_mlx_b200.synthetic import seeded_weights

    rng = np.random.default_rng(3)
    raw = _synthetic_case(rng, (1, 14, 20, 24), np.float32)
    plans = _plans((0, 1, 2), (1.0, 1.0, 1.0), ["ZScoreNormalization"], [True], {}, {"is_seg": False}, "nearest")
    result = preprocess_raw_case(raw, {"spacing": [1.0, 1.0, 1.0]}, plans, device=cuda_device)
    spec = PlainConvUNetSpec(input_channels=1, num_classes=2, features=(32, 64), kernel_sizes=((3, 3, 3),) * 2,
                             strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    net = build_network(spec, precision="fp32", device=cuda_device).load_weights(seeded_weights(spec, 0))
    on_device, _ = predict_volume([net], result.data, patch_size=(8, 16, 16), num_classes=2)
    from_host, _ = predict_volume([net], result.data.cpu().numpy(), patch_size=(8, 16, 16), num_classes=2)
    torch.testing.assert_close(on_device, from_host, rtol=1e-6, atol=1e-6)
    _status_clean()


def test_device_preprocessing_errors(cuda_device):
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case
    from nnunet_mlx_b200.errors import ContractError

    plans = _plans((0, 1, 2), (1.0, 1.0, 1.0), ["NoNormalization"], [False], {}, {"is_seg": False}, "nearest")
    with pytest.raises(ContractError, match="no nonzero"):
        preprocess_raw_case(np.zeros((1, 4, 5, 6), np.float32), {"spacing": [1, 1, 1]}, plans, device=cuda_device)
    overflow = np.zeros((1, 4, 5, 6), np.float64)
    overflow[0, 1, 1, 1] = 1e300
    with pytest.raises(ContractError, match="finite after float32"):
        preprocess_raw_case(overflow, {"spacing": [1, 1, 1]}, plans, device=cuda_device)
    rgb = _plans((0, 1, 2), (1.0, 1.0, 1.0), ["RGBTo01Normalization"], [False], {}, {"is_seg": False}, "nearest")
    bright = np.full((1, 4, 5, 6), 300.0, np.float32)
    with pytest.raises(ContractError, match=r"\[0, 255\]"):
        preprocess_raw_case(bright, {"spacing": [1, 1, 1]}, rgb, device=cuda_device)
    quadratic = PreprocessingPlans.from_payload(
        {"transpose_forward": [0, 1, 2], "configurations": {"c": {
            "spacing": [2.0, 2.0, 2.0], "normalization_schemes": ["NoNormalization"], "use_mask_for_norm": [False],
            "resampling_fn_data": "resample_data_or_seg_to_shape",
            "resampling_fn_data_kwargs": {"is_seg": False, "order": 2},
            "resampling_fn_seg": "resample_data_or_seg_to_shape", "resampling_fn_seg_kwargs": {"is_seg": True}}}},
        configuration="c")
    with pytest.raises(ContractError, match="orders 1 and 3"):
        preprocess_raw_case(np.ones((1, 4, 5, 6), np.float32), {"spacing": [1, 1, 1]}, quadratic,
                            device=cuda_device)
    with pytest.raises(ContractError, match="cascade labels"):
        preprocess_raw_case(np.ones((1, 4, 5, 6), np.float32), {"spacing": [1, 1, 1]}, quadratic,
                            segmentation_previous_stage=np.ones((1, 4, 5, 6), np.int16), device=cuda_device)
    same_grid = preprocess_raw_case(np.ones((1, 4, 5, 6), np.float32), {"spacing": [2, 2, 2]}, quadratic,
                                    device=cuda_device)
    assert tuple(same_grid.data.shape) == (1, 4, 5, 6)
    _status_clean()


@pytest.mark.parametrize("seed", range(3))
def test_device_spline_resampling_matches_scipy(cuda_device, seed):
    """Order 1 and 3, with and without a separate axis (each axis), against scipy zoom (the host path)."""
    from nnunet_mlx_b200.data.preprocessing import ResamplingContract, resample_spline_device

    rng = np.random.default_rng(200 + seed)
    for trial in range(10):
        channels = int(rng.integers(1, 3))
        source = tuple(int(v) for v in rng.integers(3, 30, 3))
        target = tuple(int(v) for v in rng.integers(2, 40, 3))
        values = (rng.standard_normal((channels, *source)) * 20).astype(np.float32)
        spacing = [float(v) for v in rng.choice([0.7, 1.0, 1.6, 3.0, 5.0], 3)]
        new = [float(v) for v in rng.choice([0.8, 1.0, 1.4, 2.5], 3)]
        order = 1 if trial % 4 == 0 else 3
        force = (None, False, True)[trial % 3]
        contract = ResamplingContract("resample_data_or_seg_to_shape", order, 0, force)
        got = resample_spline_device(torch.from_numpy(values).to(cuda_device), target, spacing, new,
                                     contract).cpu().numpy()
        expected = op.resample_spline(values, target, spacing, new, order=order, order_z=0, force_separate_z=force)
        np.testing.assert_allclose(got, expected, rtol=RTOL, atol=ATOL,
                                   err_msg=f"order {order} {source} -> {target} {spacing} -> {new}")
    _status_clean()


def test_device_preprocessing_default_spline_plan(cuda_device):
    """nnU-Net's default image resampling (order 3, separate order-0 axis) on an anisotropic CT crop."""
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case

    rng = np.random.default_rng(8)
    raw = np.zeros((1, 30, 120, 110), dtype=np.int16)
    raw[0, 1:29, 4:116, 3:107] = np.round(rng.normal(40, 200, (28, 112, 104)).clip(-1000, 3000)).astype(np.int16)
    intensity = {"0": {"mean": 100.0, "std": 50.0, "percentile_00_5": -1000.0, "percentile_99_5": 400.0}}
    plans = PreprocessingPlans.from_payload(
        {"transpose_forward": [0, 1, 2], "foreground_intensity_properties_per_channel": intensity,
         "configurations": {"c": {
             "spacing": [3.0, 1.0, 1.0], "normalization_schemes": ["CTNormalization"], "use_mask_for_norm": [False],
             "resampling_fn_data": "resample_data_or_seg_to_shape",
             "resampling_fn_data_kwargs": {"is_seg": False, "order": 3, "order_z": 0, "force_separate_z": None},
             "resampling_fn_seg": "resample_data_or_seg_to_shape",
             "resampling_fn_seg_kwargs": {"is_seg": True, "order": 1, "order_z": 0, "force_separate_z": None}}}},
        configuration="c")
    result = preprocess_raw_case(raw, {"spacing": [5.0, 0.8, 0.8]}, plans, device=cuda_device)
    reference, _, properties = op.preprocess(
        raw, [5.0, 0.8, 0.8], transpose_forward=(0, 1, 2), configured_spacing=(3.0, 1.0, 1.0),
        schemes=["CTNormalization"], use_mask=[False], intensities=intensity,
        data_resampling=dict(spline=True, order=3, order_z=0, force_separate_z=None, threshold=3.0),
        seg_resampling={})
    assert result.properties["bbox_used_for_cropping"] == properties["bbox_used_for_cropping"]
    assert tuple(result.data.shape) == reference.shape == (1, 47, 90, 83)
    np.testing.assert_allclose(result.data.cpu().numpy(), reference, rtol=RTOL, atol=ATOL)
    _status_clean()


def test_raw_case_pipeline_on_device(cuda_device, tmp_path):
    """Raw int16 case -> labels in the image's grid: device preprocessing, inference and restoration."""
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case
    from nnunet_mlx_b200.model.folder import load_model_bundle
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
    from nnunet_mlx_b200.prediction.pipeline import ModelFolderPredictor
    from nnunet_mlx_b200.synthetic import write_model_folder

    spec = PlainConvUNetSpec(input_channels=1, num_classes=3, features=(32, 64), kernel_sizes=((3, 3, 3),) * 2,
                             strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    folder = write_model_folder(tmp_path / "model", spec, seeds=(0,), patch_size=(8, 16, 16))
    plans = json.loads((folder / "plans.json").read_text())
    spline = {"order": 3, "order_z": 0, "force_separate_z": None}
    plans.update({"transpose_forward": [2, 0, 1], "transpose_backward": [1, 2, 0],
                  "foreground_intensity_properties_per_channel": {"0": {
                      "mean": 100.0, "std": 50.0, "percentile_00_5": -1000.0, "percentile_99_5": 400.0}}})
    plans["configurations"]["3d_fullres"].update({
        "spacing": [2.0, 1.0, 1.0], "normalization_schemes": ["CTNormalization"], "use_mask_for_norm": [False],
        "resampling_fn_data": "resample_data_or_seg_to_shape",
        "resampling_fn_data_kwargs": {"is_seg": False, **spline},
        "resampling_fn_seg": "resample_data_or_seg_to_shape",
        "resampling_fn_seg_kwargs": {"is_seg": True, "order": 1, "order_z": 0, "force_separate_z": None},
        "resampling_fn_probabilities": "resample_data_or_seg_to_shape",
        "resampling_fn_probabilities_kwargs": {"is_seg": False, "order": 1, "order_z": 0, "force_separate_z": None}})
    (folder / "plans.json").write_text(json.dumps(plans))
    bundle = load_model_bundle(folder, configuration="3d_fullres", device=cuda_device)
    predictor = ModelFolderPredictor(bundle)

    rng = np.random.default_rng(4)
    raw = np.zeros((1, 30, 26, 9), dtype=np.int16)
    raw[0, 2:28, 3:24, 1:8] = np.round(rng.normal(60, 150, (26, 21, 7)).clip(-1000, 2000)).astype(np.int16)
    properties = {"spacing": [0.8, 0.8, 4.0]}
    labels, prepared_properties, metrics = predictor.predict_raw_case(raw, properties, device=cuda_device)
    assert labels.shape == raw.shape[1:] and labels.dtype == np.uint16

    # the same steps one by one, restored with the host path's arithmetic (scipy zoom per plane)
    prepared = preprocess_raw_case(raw, properties, PreprocessingPlans.from_payload(plans, configuration="3d_fullres"),
                                   device=cuda_device)
    logits = predictor.predictor.predict_logits_from_preprocessed_data(prepared.data.cpu().numpy())
    crop_shape = tuple(prepared.properties["shape_after_cropping_and_before_resampling"])
    original = tuple(properties["spacing"][a] for a in (2, 0, 1))
    resampled = op.resample_spline(logits, crop_shape, (2.0, 1.0, 1.0), original, order=1, order_z=0,
                                   force_separate_z=None)
    volume = np.zeros(tuple(prepared.properties["shape_before_cropping"]), dtype=np.uint16)
    box = tuple(slice(a, b) for a, b in prepared.properties["bbox_used_for_cropping"])
    volume[box] = np.argmax(resampled, axis=0)
    expected = volume.transpose(1, 2, 0)
    ordered = np.sort(resampled, axis=0)
    clear = np.zeros(volume.shape, dtype=bool)
    clear[box] = (ordered[-1] - ordered[-2]) > 1e-4
    clear = clear.transpose(1, 2, 0)
    np.testing.assert_array_equal(labels[clear], expected[clear])
    assert (labels == expected).mean() >= 0.999
    assert prepared_properties["bbox_used_for_cropping"] == prepared.properties["bbox_used_for_cropping"]
    _status_clean()

