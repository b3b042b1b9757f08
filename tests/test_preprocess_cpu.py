"""Raw-case preprocessing on CPU: the oracle pinned against upstream's recorded vectors, and host logic.

* ``oracle/preprocess.py`` reproduces upstream ``resample_torch_fornnunet``'s recorded label
  resampling (every tie rule, interpolation mode, separate-axis policy, reference
  ``tests/test_torch_resampling.py:63-87``) and the cascade labels, bounding boxes and crop shapes
  of twelve recorded ``preprocess_raw_case`` runs (reference ``:90-117``), exactly;
* its image modes match ``torch.nn.functional.interpolate`` (upstream's implementation of the
  torch grid) within the reference's own tolerance for preprocessed data (rtol 1e-5, atol 5e-6,
  ``tests/test_torch_resampling.py:84-86``); the nearest modes exactly;
* the plans parser, new-shape rounding and the device path's refusals need no GPU.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import preprocess as op

from .conftest import GOLDEN

RTOL, ATOL = 1e-5, 5e-6


def _recorded():
    saved = np.load(GOLDEN / "torch_resampling_labels.npz")
    return saved, json.loads(str(saved["metadata"].item()))


def _oracle_kwargs(kwargs: dict) -> dict:
    return dict(mode=kwargs.get("mode", "linear"), aniso_axis_mode=kwargs.get("aniso_axis_mode", "nearest-exact"),
                force_separate_z=kwargs.get("force_separate_z"),
                threshold=kwargs.get("separate_z_anisotropy_threshold", 3.0))


def test_oracle_label_resampling_matches_upstream_recording():
    saved, meta = _recorded()
    assert len(meta["cases"]) == 72
    for case in meta["cases"]:
        kwargs = case["kwargs"]
        got = op.resample_torch(saved[f"{case['name']}-input"], case["shape"], case["spacing"], case["new_spacing"],
                                is_seg=True, tiebreak=kwargs.get("seg_tiebreak", "nearest"), **_oracle_kwargs(kwargs))
        expected = saved[f"{case['name']}-expected"]
        assert got.shape == expected.shape, case["name"]
        np.testing.assert_array_equal(got.astype(np.int64), expected.astype(np.int64), err_msg=case["name"])


def _oracle_pipeline(saved, run):
    plans = run["plans"]
    config = plans["configurations"]["selected"]
    seg = config["resampling_fn_seg_kwargs"]
    return op.preprocess(saved["raw_nonzero"].astype(np.float32), run["properties"]["spacing"],
                         transpose_forward=plans["transpose_forward"], configured_spacing=config["spacing"],
                         schemes=config["normalization_schemes"], use_mask=config["use_mask_for_norm"],
                         intensities=plans["foreground_intensity_properties_per_channel"],
                         data_resampling=_oracle_kwargs(config["resampling_fn_data_kwargs"]),
                         seg_resampling={**_oracle_kwargs(seg), "tiebreak": seg.get("seg_tiebreak", "nearest")},
                         previous=saved["previous"])


def test_oracle_preprocessing_matches_recorded_runs():
    saved, meta = _recorded()
    assert len(meta["pipeline"]) == 12
    for run in meta["pipeline"]:
        _, previous, properties = _oracle_pipeline(saved, run)
        geometry = run["geometry"]
        assert list(properties["shape_before_cropping"]) == geometry["shape_before_cropping"]
        assert properties["bbox_used_for_cropping"] == geometry["bbox_used_for_cropping"]
        assert (list(properties["shape_after_cropping_and_before_resampling"])
                == geometry["shape_after_cropping_and_before_resampling"])
        np.testing.assert_array_equal(previous.astype(np.int64), saved[f"{run['name']}-labels"].astype(np.int64),
                                      err_msg=run["name"])


@pytest.mark.parametrize("seed", range(4))
def test_oracle_image_modes_match_torch_interpolate(seed):
    rng = np.random.default_rng(seed)
    for _ in range(12):
        source = tuple(int(v) for v in rng.integers(1, 12, 3))
        target = tuple(int(v) for v in rng.integers(1, 20, 3))
        values = rng.standard_normal((2, *source)).astype(np.float32)
        tensor = torch.from_numpy(values)[None]
        linear = torch.nn.functional.interpolate(tensor, size=target, mode="trilinear", align_corners=False)[0]
        np.testing.assert_allclose(op.torch_resize(values, target, "linear", is_seg=False), linear.numpy(),
                                   rtol=RTOL, atol=ATOL)
        for mode in ("nearest", "nearest-exact"):
            reference = torch.nn.functional.interpolate(tensor, size=target, mode=mode)[0].numpy()
            np.testing.assert_array_equal(op.torch_resize(values, target, mode, is_seg=False), reference)


def test_oracle_fill_holes_bounds_ignore_enclosed_holes():
    data = np.zeros((1, 7, 8, 9), dtype=np.float32)
    data[0, 1:6, 2:7, 1:8] = 1
    data[0, 3, 4, 4] = 0  # enclosed hole
    cropped, mask, _, bounds = op.crop_to_nonzero(data, None, mask_required=True)
    assert bounds == ((1, 6), (2, 7), (1, 8))
    assert cropped.shape == (1, 5, 5, 7)
    assert (mask == 0).all()  # the hole is filled
    _, unmasked, _, _ = op.crop_to_nonzero(data, None, mask_required=False)
    assert (unmasked == 0).all()


def test_plans_parse_torch_and_spline_entries():
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, ResamplingContract

    _, meta = _recorded()
    plans = PreprocessingPlans.from_payload(meta["pipeline"][10]["plans"], configuration="selected")
    assert plans.transpose_forward == (2, 0, 1)
    assert plans.spacing == (2.5, 1.4, 0.8)
    assert plans.data_resampling.function_name == "resample_torch_fornnunet"
    assert plans.data_resampling.force_separate_z is None
    assert plans.seg_resampling.seg_tiebreak == "nearest"
    spline = ResamplingContract.from_configuration({"resampling_fn_data": "resample_data_or_seg_to_shape",
                                                    "resampling_fn_data_kwargs": {"is_seg": False}},
                                                   field="resampling_fn_data", expected_is_seg=False)
    assert (spline.order, spline.order_z, spline.force_separate_z) == (3, 0, False)


@pytest.mark.parametrize("kwargs", [{"is_seg": True}, {"is_seg": False, "mode": "cubic"},
                                    {"is_seg": False, "device": "cuda"}, {"is_seg": False, "bogus": 1},
                                    {"is_seg": False, "seg_tiebreak": "middle"}])
def test_plans_reject_bad_resampling_entries(kwargs):
    from nnunet_mlx_b200.data.preprocessing import ResamplingContract
    from nnunet_mlx_b200.errors import ContractError

    with pytest.raises(ContractError):
        ResamplingContract.from_configuration({"resampling_fn_data": "resample_torch_fornnunet",
                                               "resampling_fn_data_kwargs": kwargs},
                                              field="resampling_fn_data", expected_is_seg=False)


def test_compute_new_shape_rounds_like_python():
    from nnunet_mlx_b200.data.preprocessing import compute_new_shape

    assert compute_new_shape((7, 4, 6), (5.0, 0.7, 1.6), (2.5, 1.4, 0.8)) == (14, 2, 12)
    assert compute_new_shape((5, 5, 5), (1.0, 1.0, 1.0), (2.0, 2.0, 2.0)) == (2, 2, 2)  # round(2.5) == 2
    assert compute_new_shape((101, 768, 768), (5.0, 0.8, 0.8), (5.0, 1.0, 1.0)) == op.compute_new_shape(
        (101, 768, 768), (5.0, 0.8, 0.8), (5.0, 1.0, 1.0))


def test_device_path_refuses_before_any_launch():
    """Bad inputs raise ContractError on the host, before any device work."""
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case
    from nnunet_mlx_b200.errors import ContractError

    _, meta = _recorded()
    plans = PreprocessingPlans.from_payload(meta["pipeline"][6]["plans"], configuration="selected")
    cpu = torch.device("cpu")
    with pytest.raises(ContractError, match="CXYZ"):
        preprocess_raw_case(np.zeros((6, 8, 10), np.float32), {"spacing": [1, 1, 1]}, plans, device=cpu)
    with pytest.raises(ContractError, match="real numeric"):
        preprocess_raw_case(np.zeros((1, 6, 8, 10), np.complex64), {"spacing": [1, 1, 1]}, plans, device=cpu)
    with pytest.raises(ContractError, match="spacing"):
        preprocess_raw_case(np.zeros((1, 6, 8, 10), np.float32), {"spacing": [1, 1]}, plans, device=cpu)
    with pytest.raises(ContractError, match="normalization schemes"):
        preprocess_raw_case(np.zeros((2, 6, 8, 10), np.float32), {"spacing": [1, 1, 1]}, plans, device=cpu)
    with pytest.raises(ContractError, match="previous-stage"):
        preprocess_raw_case(np.zeros((1, 6, 8, 10), np.float32), {"spacing": [1, 1, 1]}, plans,
                            segmentation_previous_stage=np.zeros((1, 6, 8, 9), np.int16), device=cpu)


def test_oracle_nearest_axis_indices_match_reference():
    """The out-of-plane order-0 indices equal the reference's ``nearest_axis_indices`` (recorded)."""
    for case in json.loads((GOLDEN / "nearest_axis.json").read_text()):
        np.testing.assert_array_equal(op.nearest_axis_indices(case["old"], case["new"]), case["indices"])


def test_oracle_spline_separate_axis_is_planewise_zoom_then_nearest():
    """Separate-axis spline resampling = float64 per-plane zoom, then the recorded nearest indices."""
    from scipy import ndimage

    rng = np.random.default_rng(2)
    values = rng.standard_normal((1, 6, 9, 8)).astype(np.float32)
    got = op.resample_spline(values, (4, 12, 5), (5.0, 1.0, 1.0), (7.5, 0.75, 1.6), order=3, order_z=0,
                             force_separate_z=None)
    planes = [ndimage.zoom(values[0, k].astype(np.float64), (12 / 9, 5 / 8), order=3, mode="nearest",
                           grid_mode=True) for k in range(6)]
    expected = np.stack(planes)[op.nearest_axis_indices(6, 4)].astype(np.float32)
    np.testing.assert_array_equal(got[0], expected)


def test_restoration_plans_from_payload():
    from nnunet_mlx_b200.errors import ContractError
    from nnunet_mlx_b200.prediction.restore import plans_from_payload

    payload = {"transpose_forward": [2, 0, 1], "configurations": {"c": {
        "spacing": [None, 0.8, 0.8],
        "resampling_fn_probabilities": "resample_data_or_seg_to_shape",
        "resampling_fn_probabilities_kwargs": {"is_seg": False, "order": 1, "order_z": 0, "force_separate_z": None}}}}
    plans = plans_from_payload(payload, configuration="c")
    assert plans.transpose_backward == (1, 2, 0)
    assert plans.configuration.spacing == (None, 0.8, 0.8)
    entry = plans.configuration.probability_resampling
    assert (entry.function_name, entry.order, entry.order_z, entry.force_separate_z) == (
        "resample_data_or_seg_to_shape", 1, 0, None)
    with pytest.raises(ContractError, match="inverse"):
        plans_from_payload({**payload, "transpose_backward": [2, 0, 1]}, configuration="c")


def test_plan_entries_parse_like_the_reference():
    """Accept/reject decisions and parsed fields equal the reference's parser (recorded)."""
    from nnunet_mlx_b200.data.preprocessing import ResamplingContract
    from nnunet_mlx_b200.errors import ContractError

    recorded = json.loads((GOLDEN / "preprocess_policy.json").read_text())
    for entry in recorded["entries"]:
        configuration = {"f": entry["function"], "f_kwargs": entry["kwargs"]}
        expected = entry["parsed"]
        if expected is None:
            with pytest.raises(ContractError):
                ResamplingContract.from_configuration(configuration, field="f", expected_is_seg=entry["expected_is_seg"])
            continue
        parsed = ResamplingContract.from_configuration(configuration, field="f",
                                                       expected_is_seg=entry["expected_is_seg"])
        for name, value in expected.items():
            if name == "seg_tiebreak" and value is None:
                continue  # an omitted spline tie rule: only label resampling, which the device path does not do
            assert getattr(parsed, name) == value, (entry, name)


def test_new_shape_matches_reference():
    from nnunet_mlx_b200.data.preprocessing import compute_new_shape

    for case in json.loads((GOLDEN / "preprocess_policy.json").read_text())["new_shape"]:
        assert list(compute_new_shape(case["shape"], case["old"], case["new"])) == case["result"]
        assert list(op.compute_new_shape(case["shape"], case["old"], case["new"])) == case["result"]


def test_oracle_preprocessing_matches_reference_outputs():
    """Normalised data, crop boxes and cascade labels equal the reference's own ``preprocess_raw_case``."""
    saved = np.load(GOLDEN / "preprocess_reference.npz")
    cases = json.loads(str(saved["metadata"].item()))["cases"]
    assert len(cases) == 9
    for case in cases:
        plans = case["plans"]
        config = plans["configurations"]["selected"]
        name = case["name"]
        previous = saved[f"{name}-previous"] if f"{name}-previous" in saved.files else None
        data, labels, properties = op.preprocess(
            saved[f"{name}-raw"], case["spacing"], transpose_forward=plans["transpose_forward"],
            configured_spacing=config["spacing"], schemes=config["normalization_schemes"],
            use_mask=config["use_mask_for_norm"], intensities=plans["foreground_intensity_properties_per_channel"],
            data_resampling=_oracle_kwargs(config["resampling_fn_data_kwargs"]),
            seg_resampling={**_oracle_kwargs(config["resampling_fn_seg_kwargs"]), "tiebreak": "nearest"},
            previous=previous)
        assert properties["bbox_used_for_cropping"] == case["bbox"], name
        assert list(properties["shape_before_cropping"]) == case["shape_before_cropping"], name
        np.testing.assert_array_equal(data, saved[f"{name}-data"], err_msg=name)
        if previous is not None:
            np.testing.assert_array_equal(labels.astype(np.int64), saved[f"{name}-labels"].astype(np.int64),
                                          err_msg=name)


def test_plans_views_match_the_reference_parser():
    """Our preprocessing and restoration views of every recorded plans payload equal the reference's."""
    from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans
    from nnunet_mlx_b200.prediction.restore import plans_from_payload

    recorded = json.loads((GOLDEN / "plans_reference.json").read_text())
    saved, meta = _recorded()
    with np.load(GOLDEN / "preprocess_reference.npz") as reference:
        cases = json.loads(str(reference["metadata"].item()))["cases"]
    sources = {"pipeline": [run["plans"] for run in meta["pipeline"]], "reference": [c["plans"] for c in cases],
               "spline": recorded["spline_variants"]}
    assert len(recorded["parsed"]) == 24
    for expected in recorded["parsed"]:
        kind, index = expected["name"].split(":")
        payload = sources[kind][int(index)]
        ours = PreprocessingPlans.from_payload(payload, configuration="selected")
        assert list(ours.transpose_forward) == expected["transpose_forward"], expected["name"]
        assert list(ours.spacing) == expected["spacing"], expected["name"]
        assert list(ours.normalization_schemes) == expected["normalization_schemes"], expected["name"]
        assert list(ours.use_mask_for_norm) == expected["use_mask_for_norm"], expected["name"]
        for view, key in ((ours.data_resampling, "data"), (ours.seg_resampling, "seg")):
            for field, value in expected[key].items():
                assert getattr(view, field) == value, (expected["name"], key, field)
        restore = plans_from_payload(payload, configuration="selected")
        assert list(restore.transpose_backward) == expected["transpose_backward"], expected["name"]
        assert list(restore.configuration.spacing) == expected["spacing"], expected["name"]
        probabilities = restore.configuration.probability_resampling
        for field in ("function_name", "order", "order_z", "force_separate_z", "separate_z_anisotropy_threshold"):
            assert getattr(probabilities, field) == expected["probabilities"][field], (expected["name"], field)
