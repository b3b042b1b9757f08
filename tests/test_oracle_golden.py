"""Pin the CPU oracle (and the product's host geometry) to the reference's golden vectors.

The vectors in ``tests/golden`` were produced by ``tests/golden/make_golden.py``
from the reference's own host code; see that script.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import sliding_window as osw
from tests.conftest import GOLDEN


def _geometry():
    return json.loads((GOLDEN / "geometry.json").read_text())


@pytest.mark.parametrize("case", _geometry(), ids=lambda c: f"{c['image']}-{c['patch']}-{c['step']}")
def test_oracle_steps_match_reference(case):
    got = osw.compute_steps(case["image"], case["patch"], case["step"])
    assert [list(a) for a in got] == case["steps"]


@pytest.mark.parametrize("case", _geometry(), ids=lambda c: f"{c['image']}-{c['patch']}-{c['step']}")
def test_product_steps_match_reference(case):
    from nnunet_mlx_b200.prediction.sliding_window import compute_steps

    got = compute_steps(case["image"], case["patch"], step_fraction=case["step"])
    assert [list(a) for a in got] == case["steps"]


def test_baseline_tile_counts():
    # configs 2/5 (z padded to 128), 3 and 4 of the benchmark
    counts = {}
    for case in _geometry():
        n = int(np.prod([len(a) for a in case["steps"]]))
        counts[tuple(case["image"])] = n
    assert counts[(128, 768, 768)] == 121
    assert counts[(155, 240, 240)] == 18
    assert counts[(284, 400, 400)] == 144


def test_gaussian_full_match_reference():
    from nnunet_mlx_b200.prediction.sliding_window import gaussian_importance

    z = np.load(GOLDEN / "gaussian.npz")
    for key in z.files:
        if not key.startswith("full_"):
            continue
        patch = tuple(int(v) for v in key[5:].split("x"))
        np.testing.assert_array_equal(osw.gaussian_importance(patch), z[key])
        np.testing.assert_array_equal(gaussian_importance(patch), z[key])


def test_gaussian_large_patch_summary_matches_reference():
    z = np.load(GOLDEN / "gaussian.npz")
    for key in z.files:
        if not key.startswith("stats_"):
            continue
        name = key[6:]
        patch = tuple(int(v) for v in name.split("x"))
        g = osw.gaussian_importance(patch)
        c = tuple(s // 2 for s in patch)
        np.testing.assert_array_equal(g[:, c[1], c[2]], z[f"line0_{name}"])
        np.testing.assert_array_equal(g[c[0], :, c[2]], z[f"line1_{name}"])
        np.testing.assert_array_equal(g[c[0], c[1], :], z[f"line2_{name}"])
        stats = z[key]
        assert g.max() == stats[0] and g.min() == stats[1]
        assert abs(g.astype(np.float64).sum() - stats[2]) <= 1e-9 * stats[2]


def test_weight_key_mapping_matches_reference():
    from nnunet_mlx_b200.storage.weights import convert_state_dict, map_key_and_layout

    wmap = json.loads((GOLDEN / "weights_map.json").read_text())
    layouts = np.load(GOLDEN / "weights_layout.npz")
    for name, case in wmap.items():
        rng = np.random.default_rng(0)
        state = {k: rng.standard_normal(s).astype(np.float32) for k, s in case["source_shapes"].items()}
        for key, expected in case["entries"].items():
            mapped = map_key_and_layout(key, state[key])
            assert (None if mapped is None else mapped[0]) == expected, key
        converted = convert_state_dict(state)
        assert sorted(converted.weights) == case["converted_keys"]
        assert list(converted.dropped_keys) == case["dropped"]
    for key in layouts.files:
        if not key.endswith("|source"):
            continue
        name, torch_key, _ = key.split("|")
        expected = layouts[f"{name}|{torch_key}|converted"]
        got = map_key_and_layout(torch_key, layouts[key])[1]
        np.testing.assert_array_equal(got, expected)


def test_expected_shapes_match_reference_converted_keys():
    """The strict-load key set of our specs equals the reference converter's output keys."""
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec, ResidualEncoderUNetSpec
    from nnunet_mlx_b200.storage.weights import expected_shapes

    wmap = json.loads((GOLDEN / "weights_map.json").read_text())
    plain = PlainConvUNetSpec(input_channels=2, num_classes=3, features=(4, 8, 16),
                              kernel_sizes=((3, 3, 3),) * 3, strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)),
                              encoder_convs=(2, 2, 2), decoder_convs=(2, 2))
    assert sorted(expected_shapes(plain)) == wmap["plain"]["converted_keys"]
    residual = ResidualEncoderUNetSpec(input_channels=1, num_classes=3, features=(4, 8, 16),
                                       kernel_sizes=((3, 3, 3),) * 3, strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)),
                                       encoder_blocks=(1, 2, 2), decoder_convs=(1, 1))
    assert sorted(expected_shapes(residual)) == wmap["residual"]["converted_keys"]
    shapes = expected_shapes(plain)
    for torch_key, src in wmap["plain"]["source_shapes"].items():
        mlx_key = wmap["plain"]["entries"][torch_key]
        if mlx_key is None:
            continue
        if len(src) == 5:
            if mlx_key.startswith("up"):
                assert shapes[mlx_key] == (src[1], *src[2:], src[0])
            else:
                assert shapes[mlx_key] == (src[0], *src[2:], src[1])
        else:
            assert shapes[mlx_key] == tuple(src)


def test_head_argmax_matches_recorded_upstream():
    """First-argmax of recorded class logits equals upstream's recorded segmentation."""
    z = np.load(GOLDEN / "upstream_runner_subset.npz")
    logits = z["head_logits_class"]  # (C, D, H, W)
    acc = np.moveaxis(logits, 0, -1).copy()
    norm = np.ones((*acc.shape[:3], 1), np.float32)
    labels = osw.normalized_labels(acc, norm)
    np.testing.assert_array_equal(labels.astype(np.int64), z["head_segmentation_class"])


def test_oracle_mirrored_prediction_order_and_mean():
    rng = np.random.default_rng(3)
    tile = rng.standard_normal((1, 4, 5, 6, 1)).astype(np.float32)

    def model(x):
        return np.concatenate([x * 2.0, -x + 1.0], axis=-1)

    got = osw.mirrored_prediction(model, tile, (0, 1, 2))
    # pointwise model commutes with flips, so the mean of the 8 identical views is exact
    np.testing.assert_allclose(got, model(tile), rtol=1e-6, atol=1e-6)
    assert len(osw.mirror_subsets((0, 1, 2))) == 8


def test_oracle_normalized_labels_invalid_and_ties():
    acc = np.array([[[[1.0, 1.0, 0.0], [0.0, np.nan, 1.0], [2.0, 3.0, 3.0]]]], np.float32)  # (1,1,3,3)
    norm = np.array([[[[1.0], [1.0], [0.0]]]], np.float32)
    labels = osw.normalized_labels(acc, norm)
    assert labels[0, 0, 0] == 0  # tie -> first
    assert labels[0, 0, 1] == osw.INVALID_LABEL  # NaN
    assert labels[0, 0, 2] == osw.INVALID_LABEL  # zero normaliser


def test_nnunet_fp16_gaussian_matches_reference():
    """Upstream's float16 importance map (reference sliding_window.py:96-113), oracle and product."""
    from nnunet_mlx_b200.prediction.sliding_window import nnunet_fp16_gaussian

    z = np.load(GOLDEN / "gaussian.npz")
    keys = [k for k in z.files if k.startswith("fp16_")]
    assert keys
    for key in keys:
        patch = tuple(int(v) for v in key[5:].split("x"))
        assert z[key].dtype == np.float16
        np.testing.assert_array_equal(osw.nnunet_fp16_gaussian(patch), z[key])
        np.testing.assert_array_equal(nnunet_fp16_gaussian(patch), z[key])


@pytest.mark.parametrize("count", [1, 2, 3, 7])
def test_oracle_fp16_fold_rounding_matches_recorded_upstream(count):
    """Fold rounding of nnunet-fp16 (reference tests/host/test_upstream_runner_recording.py:225-246):
    each fold rounded to float16, summed in order, divided by float32(count), bitwise."""
    z = np.load(GOLDEN / "upstream_runner_subset.npz")
    folds = [z[f"rounding_input_{i}"] for i in range(count)]
    got = osw.average_folds(folds, "nnunet-fp16")
    assert got.dtype == np.float16
    np.testing.assert_array_equal(got.astype(np.float32), z[f"rounding_output_{count}"])


def test_oracle_fp16_window_is_rounded_float32_sum():
    """The fp16 window equals the half-rounded float32 sum tile by tile (single tile: exact)."""
    patch = (4, 4, 4)
    rng = np.random.default_rng(9)
    data = rng.standard_normal((1, 4, 4, 4)).astype(np.float32)

    def model(tile):
        return np.concatenate([tile, 2 * tile], axis=-1)

    got = osw.predict_logits(model, data, patch_size=patch, num_classes=2, accumulation="nnunet-fp16")
    g = osw.nnunet_fp16_gaussian(patch).astype(np.float32)
    x = np.moveaxis(data, 0, -1)
    expect_acc = np.concatenate([x, 2 * x], axis=-1) * g[..., None]
    acc16 = expect_acc.astype(np.float16)
    norm16 = g.astype(np.float16)[..., None]
    expect = (acc16.astype(np.float32) / norm16.astype(np.float32)).astype(np.float16)
    assert got.dtype == np.float16
    np.testing.assert_array_equal(got, np.moveaxis(expect, -1, 0))
