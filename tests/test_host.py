"""Host-side logic and the C-ABI library surface (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.topology import PlainConvUNetSpec, ResidualEncoderUNetSpec

ROOT = Path(__file__).resolve().parent.parent


def test_library_builds_and_exports_every_declared_symbol():
    from nnunet_mlx_b200 import _native, build

    path = build.build_extension()
    lib = ctypes.CDLL(str(path))
    header = (ROOT / "include" / "nnb.h").read_text()
    declared = set(re.findall(r"^\s*(?:int32_t|int64_t|const char\*)\s+(nnb_\w+)\(", header, re.M))
    assert declared, "no declarations found"
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in include/nnb.h but not exported"
    assert set(_native.SYMBOLS) <= declared | {"nnb_device_status"}
    assert _native.load().nnb_abi_version() == _native.ABI_VERSION


def test_plain_spec_from_plans_roundtrip(tmp_path):
    from nnunet_mlx_b200.synthetic import _plans_payload, plain_spec

    spec = plain_spec(2, 4)
    plans = _plans_payload(spec, (128, 128, 128), "3d_fullres")
    parsed = PlainConvUNetSpec.from_plans(plans, configuration="3d_fullres", input_channels=2, num_classes=4)
    assert parsed == spec


def test_residual_spec_from_plans_roundtrip():
    from nnunet_mlx_b200.synthetic import _plans_payload, resenc_spec

    spec = resenc_spec(1, 3)
    plans = _plans_payload(spec, (128, 128, 128), "3d_fullres")
    parsed = ResidualEncoderUNetSpec.from_plans(plans, configuration="3d_fullres", input_channels=1, num_classes=3)
    assert parsed == spec


@pytest.mark.parametrize("bad", [
    {"features": (32,)},
    {"kernel_sizes": ((3, 3, 3), (2, 2, 2))},
    {"leaky_slope": 1.5},
    {"norm_eps": 0.0},
    {"decoder_convs": (2, 2)},
])
def test_plain_spec_rejects_invalid(bad):
    base = dict(input_channels=1, num_classes=3, features=(4, 8), kernel_sizes=((3, 3, 3), (3, 3, 3)),
                strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    base.update(bad)
    with pytest.raises(ContractError):
        PlainConvUNetSpec(**base)


def test_plans_reject_unsupported_ops():
    from nnunet_mlx_b200.synthetic import _plans_payload, plain_spec

    plans = _plans_payload(plain_spec(1, 3), (128, 128, 128), "3d_fullres")
    arch = plans["configurations"]["3d_fullres"]["architecture"]["arch_kwargs"]
    arch["norm_op"] = "torch.nn.BatchNorm3d"
    with pytest.raises(ContractError):
        PlainConvUNetSpec.from_plans(plans, configuration="3d_fullres", input_channels=1, num_classes=3)


def test_seeded_weights_are_deterministic_and_complete():
    from nnunet_mlx_b200.storage.weights import expected_shapes, validate_weights
    from nnunet_mlx_b200.synthetic import config_spec, seeded_weights

    spec = config_spec(1)
    a, b = seeded_weights(spec, 0), seeded_weights(spec, 0)
    assert set(a) == set(expected_shapes(spec))
    for key in a:
        np.testing.assert_array_equal(a[key], b[key])
    validate_weights(spec, a)
    params = sum(v.size for v in a.values())
    assert 30e6 < params < 32e6  # ~31.2 M parameters (all seg heads included)


def test_resenc_parameter_count():
    from nnunet_mlx_b200.storage.weights import expected_shapes
    from nnunet_mlx_b200.synthetic import config_spec

    params = sum(int(np.prod(s)) for s in expected_shapes(config_spec(5)).values())
    assert 100e6 < params < 105e6


def test_validate_weights_strict():
    from nnunet_mlx_b200.storage.weights import validate_weights
    from nnunet_mlx_b200.synthetic import plain_spec, seeded_weights

    spec = plain_spec(1, 3, features=(4, 8), patch_stages=2)
    weights = seeded_weights(spec, 1)
    broken = dict(weights)
    broken.pop("seg0.bias")
    with pytest.raises(ContractError):
        validate_weights(spec, broken)
    bad = dict(weights)
    bad["enc0.block0.conv.weight"] = bad["enc0.block0.conv.weight"][..., :0]
    with pytest.raises(ContractError):
        validate_weights(spec, bad)
    nan = dict(weights)
    nan["enc1.block0.norm.weight"] = np.full_like(nan["enc1.block0.norm.weight"], np.nan)
    with pytest.raises(ContractError):
        validate_weights(spec, nan)


def test_model_folder_roundtrip(tmp_path):
    from nnunet_mlx_b200.storage.checkpoint import load_inference_checkpoint
    from nnunet_mlx_b200.synthetic import plain_spec, seeded_weights, write_model_folder

    spec = plain_spec(1, 3, features=(4, 8), patch_stages=2)
    folder = write_model_folder(tmp_path / "model", spec, seeds=(3, 4), patch_size=(16, 16, 16))
    state, weights = load_inference_checkpoint(folder / "fold_1" / "checkpoint_final")
    assert state.identity.fold == 1
    assert state.inference_allowed_mirroring_axes == (0, 1, 2)
    ref = seeded_weights(spec, 4)
    for key in ref:
        np.testing.assert_array_equal(weights[key], ref[key])
    (folder / "fold_0" / "checkpoint_final" / "extra.bin").write_bytes(b"x")
    with pytest.raises(ContractError):
        load_inference_checkpoint(folder / "fold_0" / "checkpoint_final")


def test_mirror_masks_follow_reference_view_order():
    from nnunet_mlx_b200.prediction.sliding_window import mirror_masks

    assert mirror_masks((0, 1, 2)) == [0, 1, 2, 4, 3, 5, 6, 7]
    assert mirror_masks((1, 2)) == [0, 2, 4, 6]
    assert mirror_masks(()) == [0]


def test_pad_minimum_matches_oracle():
    from oracle.sliding_window import pad_minimum as opad

    from nnunet_mlx_b200.prediction.sliding_window import pad_minimum

    data = np.zeros((1, 5, 130, 7), np.float32)
    padded, crop = opad(data, (8, 128, 8))
    pads, crop2 = pad_minimum(data.shape[1:], (8, 128, 8))
    assert crop == crop2
    assert tuple(s + a + b for s, (a, b) in zip(data.shape[1:], pads)) == padded.shape[1:]


def test_synthetic_volumes_have_config_shapes_and_ranges():
    from nnunet_mlx_b200.synthetic import ct_normalize, synthetic_ct_hu

    hu = synthetic_ct_hu((16, 64, 64), seed=1)
    assert hu.dtype == np.int16
    assert (hu < -900).mean() > 0.3  # mostly air
    x = ct_normalize(hu)
    assert x.min() >= (-1000 - 100) / 50 and x.max() <= (400 - 100) / 50


def _conv_args(cins, cout, dims, kernel, stride, pad, precision):
    from nnunet_mlx_b200 import _native

    args = _native.Conv3dArgs()
    args.batch = 2
    args.in_dims = _native.dims3(dims)
    args.out_dims = _native.dims3(tuple((d + 2 * p - k) // s + 1 for d, p, k, s in zip(dims, pad, kernel, stride)))
    args.kernel = _native.dims3(kernel)
    args.stride = _native.dims3(stride)
    args.pad = _native.dims3(pad)
    args.num_segments = len(cins)
    for i, c in enumerate(cins):
        args.seg[i] = _native.Segment(0, 0, 0, c, 1)
    args.cout = cout
    args.precision = precision
    return args


@pytest.mark.parametrize("cins,cout,dims,kernel,stride,pad,precision,expect", [
    ((32,), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 1),     # z-streaming, resident weights
    ((32, 32), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 1),  # concat, streamed weights
    ((32,), 16, (4, 8, 8), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 1),
    ((32,), 64, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 0),     # > 32 output channels
    ((32,), 32, (16, 16, 16), (3, 3, 3), (2, 2, 2), (1, 1, 1), 0, 0),     # strided
    ((32,), 32, (16, 16, 16), (1, 3, 3), (1, 1, 1), (0, 1, 1), 0, 0),     # anisotropic kernel
    ((32,), 32, (16, 4, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 0),      # rows shorter than a brick
    ((32,), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 3, 0),     # split-TF32 fallback precision
    ((32,), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 1, 1),     # TF32 z-streaming
    ((32,), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 4, 1),     # BF16 z-streaming
    ((32, 32), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 4, 1),  # BF16 concat, resident weights
    ((64,), 64, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 4, 0),     # BF16, > 32 output channels
    ((16,), 32, (16, 16, 16), (3, 3, 3), (1, 1, 1), (1, 1, 1), 0, 0),     # channels not a multiple of 32
])
def test_raw_operand_query(cins, cout, dims, kernel, stride, pad, precision, expect):
    """Which layers the tensor-core path reads as raw lazy activations (no device work: shape logic only)."""
    from nnunet_mlx_b200 import _native

    args = _conv_args(cins, cout, dims, kernel, stride, pad, precision)
    assert _native.load().nnb_conv3d_raw_operands(ctypes.byref(args)) == expect
