"""Network forward and sliding-window parity on B200 against the CPU oracle.

Tolerance (the path's parity bar): logits within rel 1e-3 / abs 1e-3 of the float32
oracle in the default ("fp32": split fp16-pair tensor cores) mode and in its
split-TF32 range fallback ("fp32-tf32x2"), argmax agreement >= 99.95% with
disagreements only at near-ties.  The single-pass TF32 fast mode is checked
against its own stated, looser bound.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import network as onet
from oracle import sliding_window as osw

pytestmark = pytest.mark.gpu

LOGIT_TOL = dict(rtol=1e-3, atol=1e-3)


def _spec(kind: str):
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec, ResidualEncoderUNetSpec

    k3 = (3, 3, 3)
    if kind == "tiny":
        return PlainConvUNetSpec(input_channels=1, num_classes=3, features=(4, 8), kernel_sizes=(k3, k3),
                                 strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    if kind == "tiny_residual":
        return ResidualEncoderUNetSpec(input_channels=1, num_classes=3, features=(4, 8, 16), kernel_sizes=(k3,) * 3,
                                       strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)), encoder_blocks=(1, 3, 4),
                                       decoder_convs=(1, 1))
    if kind == "tiny_bottleneck":
        return ResidualEncoderUNetSpec(input_channels=1, num_classes=3, features=(4, 8, 16), kernel_sizes=(k3,) * 3,
                                       strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)), encoder_blocks=(1, 2, 2),
                                       decoder_convs=(1, 1), bottleneck_channels=(2, 4, 8))
    if kind == "mid":
        return PlainConvUNetSpec(input_channels=2, num_classes=4, features=(32, 64, 128), kernel_sizes=(k3,) * 3,
                                 strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)), encoder_convs=(2, 2, 2),
                                 decoder_convs=(2, 2))
    if kind == "mid_residual":
        return ResidualEncoderUNetSpec(input_channels=1, num_classes=3, features=(32, 64, 64),
                                       kernel_sizes=(k3,) * 3, strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)),
                                       encoder_blocks=(1, 2, 2), decoder_convs=(1, 1))
    if kind == "anisotropic":
        return PlainConvUNetSpec(input_channels=1, num_classes=2, features=(32, 64, 96),
                                 kernel_sizes=((1, 3, 3), (3, 3, 3), (3, 3, 3)),
                                 strides=((1, 1, 1), (1, 2, 2), (2, 2, 2)), encoder_convs=(2, 2, 2),
                                 decoder_convs=(1, 1))
    raise KeyError(kind)


def _network(spec, seed, device, precision="fp32"):
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.synthetic import seeded_weights

    weights = seeded_weights(spec, seed)
    # non-trivial norm affine and biases so their handling is exercised
    rng = np.random.default_rng(seed + 100)
    for key in weights:
        if key.endswith("norm.weight"):
            weights[key] = rng.uniform(0.5, 1.5, weights[key].shape).astype(np.float32)
        elif key.endswith("bias"):
            weights[key] = (0.1 * rng.standard_normal(weights[key].shape)).astype(np.float32)
    net = build_network(spec, precision=precision, device=device).load_weights(weights)
    return net, weights


def _assert_logits(got, ref, tol=LOGIT_TOL, argmax_min=0.9995):
    np.testing.assert_allclose(got, ref, **tol)
    agree = (got.argmax(-1) == ref.argmax(-1)).mean()
    assert agree >= argmax_min, agree


@pytest.mark.parametrize("kind,shape", [
    ("tiny", (2, 8, 12, 10)),
    ("tiny_residual", (2, 16, 16, 8)),
    ("tiny_bottleneck", (1, 8, 8, 16)),
    ("mid", (2, 16, 16, 16)),
    ("mid_residual", (2, 16, 24, 16)),
    ("anisotropic", (1, 8, 16, 16)),
])
def test_forward_matches_oracle(cuda_device, kind, shape):
    spec = _spec(kind)
    net, weights = _network(spec, 3, cuda_device)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((shape[0], *shape[1:], spec.input_channels)).astype(np.float32)
    got = net(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    ref = onet.forward(x, weights, spec)
    _assert_logits(got, ref)


@pytest.mark.parametrize("precision", ["fp32", "fp32-tf32x2"])
def test_full_network_forward_64_matches_oracle(cuda_device, precision):
    """The benchmark network (6 stages, 32..320) on a 64^3 synthetic CT tile."""
    from nnunet_mlx_b200.synthetic import config_spec, synthetic_ct

    spec = config_spec(1)
    net, weights = _network(spec, 0, cuda_device, precision=precision)
    x = np.moveaxis(synthetic_ct((64, 96, 96), seed=1)[:, :, :64, :64], 0, -1)[None].copy()
    got = net(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    ref = onet.forward(x, weights, spec)
    _assert_logits(got, ref)


def test_tf32_fast_mode_stated_bound(cuda_device):
    """Single-pass TF32: stated bound max |err| <= 0.25 (logits of magnitude ~O(5)), argmax >= 98%."""
    from nnunet_mlx_b200.synthetic import config_spec, synthetic_ct

    spec = config_spec(1)
    net, weights = _network(spec, 0, cuda_device, precision="tf32")
    x = np.moveaxis(synthetic_ct((64, 96, 96), seed=1)[:, :, :64, :64], 0, -1)[None].copy()
    got = net(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    ref = onet.forward(x, weights, spec)
    assert np.abs(got - ref).max() <= 0.25
    assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.98


def _oracle_model(weights, spec):
    return lambda tile: onet.forward(tile, weights, spec)


@pytest.mark.parametrize("shape,patch,axes", [
    ((1, 17, 33, 49), (16, 32, 32), (0, 1, 2)),
    ((1, 5, 6, 7), (4, 4, 4), ()),
    ((1, 9, 14, 3), (8, 8, 8), (1, 2)),   # an axis shorter than the patch (padding + crop)
])
def test_sliding_window_matches_oracle(cuda_device, shape, patch, axes):
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec = _spec("tiny")
    net, weights = _network(spec, 5, cuda_device)
    data = np.random.default_rng(12).standard_normal(shape).astype(np.float32)
    logits, labels = predict_volume([net], data, patch_size=patch, num_classes=3, mirroring_axes=axes)
    ref = osw.predict_logits(_oracle_model(weights, spec), data, patch_size=patch, num_classes=3,
                             mirroring_axes=axes)
    got = logits.cpu().numpy()
    np.testing.assert_allclose(got, ref, **LOGIT_TOL)
    assert (labels.cpu().numpy() == ref.argmax(0)).mean() >= 0.9995


def test_fold_ensemble_matches_oracle(cuda_device):
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec = _spec("tiny")
    nets = [_network(spec, seed, cuda_device) for seed in (21, 22)]
    data = np.random.default_rng(13).standard_normal((1, 12, 20, 18)).astype(np.float32)
    logits, _ = predict_volume([n for n, _ in nets], data, patch_size=(8, 16, 16), num_classes=3,
                               mirroring_axes=(0, 2))
    ref = osw.average_fold_logits([_oracle_model(w, spec) for _, w in nets], data, patch_size=(8, 16, 16),
                                  num_outputs=3, mirroring_axes=(0, 2))
    np.testing.assert_allclose(logits.cpu().numpy(), ref, **LOGIT_TOL)


def test_mid_network_sliding_window_tensor_cores(cuda_device):
    """Tensor-core layers inside the sliding window, 8 mirrored views per tile."""
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec = _spec("mid")
    net, weights = _network(spec, 7, cuda_device)
    data = np.random.default_rng(14).standard_normal((2, 20, 24, 18)).astype(np.float32)
    logits, labels = predict_volume([net], data, patch_size=(16, 16, 16), num_classes=4, mirroring_axes=(0, 1, 2))
    ref = osw.predict_logits(_oracle_model(weights, spec), data, patch_size=(16, 16, 16), num_classes=4,
                             mirroring_axes=(0, 1, 2))
    np.testing.assert_allclose(logits.cpu().numpy(), ref, **LOGIT_TOL)
    assert (labels.cpu().numpy() == ref.argmax(0)).mean() >= 0.9995


def test_fp32_range_fallback_recomputes_in_split_tf32(cuda_device):
    """An activation beyond the fp16-pair range (norm gain 2e5) sends the volume to the split-TF32 twin."""
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec = _spec("mid")
    net, weights = _network(spec, 8, cuda_device)
    weights["enc0.block0.norm.weight"] = np.full_like(weights["enc0.block0.norm.weight"], 2e5)
    net = build_network(spec, precision="fp32", device=cuda_device).load_weights(weights)
    twin = build_network(spec, precision="fp32-tf32x2", device=cuda_device).load_weights(weights)
    data = np.random.default_rng(15).standard_normal((2, 16, 20, 16)).astype(np.float32)
    args = dict(patch_size=(16, 16, 16), num_classes=4, mirroring_axes=(0, 2))
    logits, labels = predict_volume([net], data, **args)
    assert net._fallback is not None, "the range guard did not fire"
    ref_logits, ref_labels = predict_volume([twin], data, **args)
    assert twin._fallback is None
    np.testing.assert_array_equal(logits.cpu().numpy(), ref_logits.cpu().numpy())
    np.testing.assert_array_equal(labels.cpu().numpy(), ref_labels.cpu().numpy())
    ref = osw.predict_logits(_oracle_model(weights, spec), data, num_classes=4, patch_size=(16, 16, 16),
                             mirroring_axes=(0, 2))
    np.testing.assert_allclose(logits.cpu().numpy(), ref, **LOGIT_TOL)


def test_fp32_mode_stays_on_fp16_pairs_for_normalised_activations(cuda_device):
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec = _spec("mid")
    net, _ = _network(spec, 9, cuda_device)
    data = np.random.default_rng(16).standard_normal((2, 16, 16, 16)).astype(np.float32)
    predict_volume([net], data, patch_size=(16, 16, 16), num_classes=4, mirroring_axes=(0,))
    assert net._fallback is None
