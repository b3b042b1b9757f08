"""nnunet-fp16 accumulation on B200: the device fold kernels against upstream's recorded
float16 fold-rounding vectors (bitwise), and the float16 sliding window against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import network as onet
from oracle import sliding_window as osw
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("count", [1, 2, 3, 7])
def test_device_fold_rounding_matches_recorded_upstream(cuda_device, count):
    """Folds enter as float16 windows with a unit normaliser, so each normalised fold is
    half(input); fold_add sums them in order and fold_finalize divides: bitwise vs upstream."""
    from nnunet_mlx_b200 import kernels

    z = np.load(GOLDEN / "upstream_runner_subset.npz")
    classes, *dims = z["rounding_input_0"].shape
    total = torch.empty((classes, *dims), dtype=torch.float16, device=cuda_device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    norm = torch.ones(tuple(dims), dtype=torch.float16, device=cuda_device)
    for i in range(count):
        fold = np.moveaxis(z[f"rounding_input_{i}"], 0, -1).astype(np.float16)  # channels-last half window
        acc = torch.from_numpy(np.ascontiguousarray(fold)).to(cuda_device)
        kernels.fold_add_fp16(acc, norm, (0, 0, 0), dims, total, i == 0, invalid)
    logits, labels, bad = kernels.fold_finalize_fp16(total, count, label_dtype=torch.uint8)
    assert int(invalid.item()) == 0 and int(bad.item()) == 0
    expect = z[f"rounding_output_{count}"]
    np.testing.assert_array_equal(logits.cpu().numpy(), expect)
    np.testing.assert_array_equal(total.cpu().numpy().astype(np.float32), expect)
    np.testing.assert_array_equal(labels.cpu().numpy(), expect.argmax(0))


def _tiny(seed, device):
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
    from nnunet_mlx_b200.synthetic import seeded_weights

    k3 = (3, 3, 3)
    spec = PlainConvUNetSpec(input_channels=1, num_classes=3, features=(4, 8), kernel_sizes=(k3, k3),
                             strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    weights = seeded_weights(spec, seed)
    return build_network(spec, precision="fp32", device=device).load_weights(weights), weights, spec


def _ulp16(x):
    return np.spacing(np.abs(x).astype(np.float16)).astype(np.float32)


@pytest.mark.parametrize("folds", [1, 2])
def test_fp16_window_fold_kernels_bitwise_on_exact_predictions(cuda_device, folds):
    """Integer features and head weights make every view's logits, their sum and the /8 view mean
    exact in float32 on both sides, and pred * g is exact too; the float16 window updates over
    overlapping tiles, the per-fold normalisation, fold sum and divide must then match the oracle's
    float16 arithmetic bitwise."""
    from nnunet_mlx_b200 import kernels
    from nnunet_mlx_b200.kernels import Lazy
    from nnunet_mlx_b200.prediction.sliding_window import mirror_masks, nnunet_fp16_gaussian

    rng = np.random.default_rng(40 + folds)
    patch, classes, feats = (4, 6, 8), 3, 32
    masks = mirror_masks((0, 1, 2))
    views = len(masks)
    vol = (7, 9, 12)
    offsets = [(0, 0, 0), (2, 1, 3), (3, 3, 4), (1, 3, 0)]
    g16 = nnunet_fp16_gaussian(patch)
    g32 = g16.astype(np.float32)
    gaussian = torch.from_numpy(np.ascontiguousarray(g32)).to(cuda_device)
    total = torch.empty((classes, *vol), dtype=torch.float16, device=cuda_device)
    invalid = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    ref_total = None
    for f in range(folds):
        acc = torch.zeros((*vol, classes), dtype=torch.float16, device=cuda_device)
        nrm = torch.zeros(vol, dtype=torch.float16, device=cuda_device)
        ref_acc = np.zeros((*vol, classes), np.float16)
        ref_nrm = np.zeros(vol, np.float16)
        wseg = rng.integers(-1, 2, (classes, feats)).astype(np.float32)
        bseg = rng.integers(-2, 3, classes).astype(np.float32)
        w_dev, b_dev = torch.from_numpy(wseg).to(cuda_device), torch.from_numpy(bseg).to(cuda_device)
        for off in offsets:
            x = rng.integers(-2, 3, (views, *patch, feats)).astype(np.float32)
            kernels.accumulate_tile(Lazy(torch.from_numpy(x).to(cuda_device)), masks, w_dev, b_dev, gaussian, acc,
                                    nrm, off, True, 0.01)
            logits = x @ wseg.T + bseg
            pred = logits[0].copy()
            for v in range(1, views):
                pred = pred + np.flip(logits[v], axis=tuple(a for a in range(3) if masks[v] >> a & 1))
            pred = (pred / np.float32(views)).astype(np.float32)
            sl = tuple(slice(o, o + p) for o, p in zip(off, patch))
            ref_acc[sl] = (ref_acc[sl].astype(np.float32) + pred * g32[..., None]).astype(np.float16)
            ref_nrm[sl] = (ref_nrm[sl].astype(np.float32) + g32).astype(np.float16)
        np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
        np.testing.assert_array_equal(nrm.cpu().numpy(), ref_nrm)
        # the crop covers the whole window; voxels no tile touched have a zero normaliser (non-finite)
        covered = ref_nrm > 0
        kernels.fold_add_fp16(acc, nrm, (0, 0, 0), vol, total, f == 0, invalid)
        with np.errstate(divide="ignore", invalid="ignore"):
            fold = (ref_acc.astype(np.float32) / ref_nrm.astype(np.float32)[..., None]).astype(np.float16)
        fold = np.moveaxis(fold, -1, 0)
        ref_total = fold if ref_total is None else (ref_total.astype(np.float32) +
                                                    fold.astype(np.float32)).astype(np.float16)
    assert int(invalid.item()) == folds * int((~covered).sum())
    logits, labels, bad = kernels.fold_finalize_fp16(total, folds, label_dtype=torch.uint8)
    ref_avg = (ref_total.astype(np.float32) / np.float32(folds)).astype(np.float16)
    got = logits.cpu().numpy()
    np.testing.assert_array_equal(got[:, covered], ref_avg.astype(np.float32)[:, covered])
    np.testing.assert_array_equal(labels.cpu().numpy()[covered], ref_avg.astype(np.float32).argmax(0)[covered])
    assert (labels.cpu().numpy()[~covered] == 255).all()
    assert int(bad.item()) == int((~covered).sum())


def _assert_fp16_close(got, ref):
    """Device network outputs differ from the float32 CPU oracle's by float32 rounding (~1e-6 rel), so a
    float16 window update can round to the neighbouring half value; such a flip moves a normalised
    logit by one half ulp of the accumulated window value / normaliser -- a few 1e-4 for unit-scale
    logits.  Almost all values must match bitwise."""
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    diff = np.abs(got - ref)
    assert (diff <= 8 * _ulp16(np.maximum(np.abs(ref), 1.0))).all(), diff.max()
    assert (diff == 0).mean() >= 0.95, (diff == 0).mean()


def test_fp16_sliding_window_fold_ensemble_matches_oracle(cuda_device):
    """Two folds, mirroring, padding + crop: float16 logits against the oracle's float16 mode,
    labels agreeing."""
    from nnunet_mlx_b200.prediction.inference import average_fold_logits

    nets = [_tiny(seed, cuda_device) for seed in (31, 32)]
    data = np.random.default_rng(15).standard_normal((1, 12, 20, 7)).astype(np.float32)
    patch = (8, 16, 8)
    got = average_fold_logits([n for n, _, _ in nets], data, patch_size=patch, num_outputs=3,
                              mirroring_axes=(0, 1, 2), accumulation="nnunet-fp16")
    ref = osw.average_fold_logits([(lambda t, w=w, s=s: onet.forward(t, w, s)) for _, w, s in nets], data,
                                  patch_size=patch, num_outputs=3, mirroring_axes=(0, 1, 2),
                                  accumulation="nnunet-fp16")
    assert got.dtype == np.float16 and ref.dtype == np.float16 and got.shape == ref.shape
    _assert_fp16_close(got, ref)
    assert (got.astype(np.float32).argmax(0) == ref.astype(np.float32).argmax(0)).mean() >= 0.999


def test_fp16_labels_and_device_logits(cuda_device):
    from nnunet_mlx_b200.prediction.sliding_window import predict_device_logits, predict_labels, predict_logits

    net, weights, spec = _tiny(33, cuda_device)
    data = np.random.default_rng(16).standard_normal((1, 9, 17, 16)).astype(np.float32)
    kw = dict(patch_size=(8, 8, 8), num_classes=3, mirroring_axes=(1,), accumulation="nnunet-fp16")
    host = predict_logits(net, data, **kw)
    device = predict_device_logits(net, data, **kw)
    labels = predict_labels(net, data, **kw)
    assert host.dtype == np.float32 and device.dtype == torch.float16
    np.testing.assert_array_equal(host, np.moveaxis(device.float().cpu().numpy(), -1, 0))
    np.testing.assert_array_equal(labels, host.argmax(0))
    ref = osw.predict_logits(lambda t: onet.forward(t, weights, spec), data, **kw)
    _assert_fp16_close(host, ref)
