"""Parity at the benchmark sizes: the CUDA path against the CPU oracle on the benchmark networks.

* Configuration 1 exactly: the 6-stage PlainConvUNet (32..320), seed-0
  Kaiming weights, gamma = 1, beta = 0, zero biases, one 128^3 N(0, 1) tile
  from ``default_rng(0)``, no mirroring (reference parity shapes:
  ``tests/test_torch_oracle_parity.py:136-161``).
* The configuration-5 ResEnc-L network (blocks (1, 3, 4, 6, 6, 6), seed 30)
  on a 128^3 crop of the configuration-2 CT.
* An 8-view sliding window with the full configuration-2 network over a
  101 x 192 x 192 crop of the configuration-2 CT: z = 101 is padded to the
  128 patch as in configuration 2, and 2 x 2 tiles overlap in y and x
  (reference ``tests/test_torch_oracle_parity.py:186-207``).

Tolerances: the default ``fp32`` mode must keep logits within rel/abs 1e-3
of the float32 oracle and argmax agreement >= 99.95%, and every disagreement
must be a near-tie (the oracle's top-two gap below the logit tolerance).  The
single-pass ``tf32`` and ``bf16`` modes are held to the looser bounds stated
beside them; each test prints the measured figures (``-s``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import network as onet
from oracle import sliding_window as osw

pytestmark = pytest.mark.gpu

LOGIT_TOL = dict(rtol=1e-3, atol=1e-3)
# Stated bounds of the single-pass modes on the benchmark networks (measured on B200 against the
# float32 oracle; the figures each test prints are recorded in the design notes).
# Measured: tf32 max|err| 0.014 (window) / 0.026 (ResEnc-L), argmax 99.85%; bf16 0.096 / 0.21, argmax 98.85%.
LOOSE_BOUNDS = {
    "tf32": {"max_abs": 0.1, "argmax": 0.995},
    "bf16": {"max_abs": 0.5, "argmax": 0.98},
}


def assert_parity(got: np.ndarray, ref: np.ndarray, axis: int, label: str) -> None:
    """rel/abs 1e-3 logits, >= 99.95% argmax agreement, disagreements only at near-ties."""
    np.testing.assert_allclose(got, ref, **LOGIT_TOL)
    g, r = got.argmax(axis), ref.argmax(axis)
    agree = float((g == r).mean())
    top = np.sort(ref, axis=axis)
    first = np.take(top, -1, axis=axis)
    gap = first - np.take(top, -2, axis=axis)
    bound = 2.0 * (LOGIT_TOL["atol"] + LOGIT_TOL["rtol"] * np.abs(first))
    ties = gap[g != r]
    print(f"PARITY {label}: max|err| {np.abs(got - ref).max():.3g} argmax {agree:.6f} "
          f"disagreements {int((g != r).sum())} (largest top-2 gap {ties.max() if ties.size else 0:.3g})")
    assert agree >= 0.9995, agree
    assert (ties <= bound[g != r]).all(), "an argmax disagreement is not a near-tie"


def assert_loose(got: np.ndarray, ref: np.ndarray, axis: int, precision: str, label: str) -> None:
    err = float(np.abs(got - ref).max())
    agree = float((got.argmax(axis) == ref.argmax(axis)).mean())
    close = float(np.isclose(got, ref, **LOGIT_TOL).mean())
    print(f"BOUND {label} {precision}: max|err| {err:.4g} argmax {agree:.6f} within-1e-3 {close:.4f}")
    bound = LOOSE_BOUNDS[precision]
    assert err <= bound["max_abs"], err
    assert agree >= bound["argmax"], agree


def _net(spec, weights, device, precision):
    from nnunet_mlx_b200.model.network import build_network

    return build_network(spec, precision=precision, device=device).load_weights(weights)


@pytest.fixture(scope="module")
def ct_volume():
    from nnunet_mlx_b200.synthetic import synthetic_ct

    return synthetic_ct()  # (1, 101, 768, 768), the configuration-2 CT


@pytest.fixture(scope="module")
def config1():
    from nnunet_mlx_b200.synthetic import config_spec, config_volume, seeded_weights

    spec = config_spec(1)
    weights = seeded_weights(spec, 0)
    x = np.moveaxis(config_volume(1), 0, -1)[None].copy()  # (1, 128, 128, 128, 1)
    return spec, weights, x, onet.forward(x, weights, spec)


@pytest.fixture(scope="module")
def config5(ct_volume):
    from nnunet_mlx_b200.synthetic import config_spec, seeded_weights

    spec = config_spec(5)
    weights = seeded_weights(spec, 30)
    # 128^3: the 101 CT planes zero-padded to 128 (as the window pads them), centre 128^2 in-plane
    crop = np.zeros((1, 128, 128, 128), np.float32)
    crop[:, 13:114] = ct_volume[:, :, 320:448, 320:448]
    x = np.moveaxis(crop, 0, -1)[None].copy()
    return spec, weights, x, onet.forward(x, weights, spec)


@pytest.fixture(scope="module")
def window2(ct_volume):
    from nnunet_mlx_b200.synthetic import config_spec, seeded_weights

    spec = config_spec(2)
    weights = seeded_weights(spec, 0)
    data = np.ascontiguousarray(ct_volume[:, :, 288:480, 288:480])  # (1, 101, 192, 192): 4 tiles of 128^3
    ref = osw.predict_logits(lambda t: onet.forward(t, weights, spec), data, patch_size=(128, 128, 128),
                             num_classes=3, mirroring_axes=(0, 1, 2))
    return spec, weights, data, ref


def test_config1_forward_matches_oracle(cuda_device, config1):
    spec, weights, x, ref = config1
    got = _net(spec, weights, cuda_device, "fp32")(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert_parity(got, ref, -1, "config1 128^3 forward")


def test_resenc_l_forward_matches_oracle(cuda_device, config5):
    spec, weights, x, ref = config5
    got = _net(spec, weights, cuda_device, "fp32")(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert_parity(got, ref, -1, "config5 ResEnc-L 128^3 forward")


def test_config2_window_matches_oracle(cuda_device, window2):
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec, weights, data, ref = window2
    net = _net(spec, weights, cuda_device, "fp32")
    logits, labels = predict_volume([net], data, patch_size=(128, 128, 128), num_classes=3,
                                    mirroring_axes=(0, 1, 2))
    got = logits.cpu().numpy()
    assert_parity(got, ref, 0, "config2 crop 8-view window")
    assert (labels.cpu().numpy() == got.argmax(0)).all()


@pytest.mark.parametrize("precision", ["tf32", "bf16"])
def test_loose_modes_config2_window(cuda_device, window2, precision):
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    spec, weights, data, ref = window2
    net = _net(spec, weights, cuda_device, precision)
    logits, _ = predict_volume([net], data, patch_size=(128, 128, 128), num_classes=3, mirroring_axes=(0, 1, 2))
    assert_loose(logits.cpu().numpy(), ref, 0, precision, "config2 crop 8-view window")


@pytest.mark.parametrize("precision", ["tf32", "bf16"])
def test_loose_modes_config5_forward(cuda_device, config5, precision):
    spec, weights, x, ref = config5
    got = _net(spec, weights, cuda_device, precision)(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert_loose(got, ref, -1, precision, "config5 ResEnc-L 128^3 forward")
