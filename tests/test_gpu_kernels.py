"""Per-kernel parity on B200: every C-ABI compute entry point against the CPU oracle.

The oracle side is plain PyTorch-CPU float32 (``torch.nn.functional``) or
NumPy restating the reference semantics; tolerances are written per test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

FP32_TOL = dict(rtol=2e-4, atol=2e-4)     # split fp16 pairs / split TF32 / CUDA-core float32 vs float32 reference
TF32_TOL = dict(rtol=2e-2, atol=2e-2)     # single-pass TF32 (fast mode)


def _lazy_ref(raw, scale, shift, leaky, slope=0.01):
    """Reference activation of a lazy segment: (B, D, H, W, C) numpy-like torch CPU."""
    if scale is None:
        return raw
    y = raw * scale[:, None, None, None, :] + shift[:, None, None, None, :]
    return F.leaky_relu(y, slope) if leaky else y


def _conv_ref(parts, weight, stride, pad, bias=None):
    x = torch.cat(parts, dim=-1).permute(0, 4, 1, 2, 3)
    w = weight.permute(0, 4, 1, 2, 3)
    y = F.conv3d(x.double(), w.double(), None if bias is None else bias.double(), stride=stride, padding=pad)
    return y.permute(0, 2, 3, 4, 1).float()


def _make_segment(rng, batch, dims, channels, lazy, device):
    from nnunet_mlx_b200.kernels import Lazy

    raw = torch.from_numpy(rng.standard_normal((batch, *dims, channels)).astype(np.float32) * 2 + 0.5)
    if not lazy:
        return Lazy(raw.to(device)), raw, None, None
    scale = torch.from_numpy(rng.uniform(0.5, 1.5, (batch, channels)).astype(np.float32))
    shift = torch.from_numpy(rng.standard_normal((batch, channels)).astype(np.float32))
    return Lazy(raw.to(device), scale.to(device), shift.to(device), leaky=True), raw, scale, shift


CONV_CASES = [
    # (batch, in_dims, segments [(channels, lazy)], cout, kernel, stride, pad, precision)
    (2, (6, 7, 9), [(1, False)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "simt"),
    # first-layer kernel (persistent blocks looping over tiles, partial last tile, two channel groups)
    (3, (33, 40, 47), [(1, False)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "simt"),
    (2, (17, 20, 23), [(2, False)], 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "simt"),
    (1, (9, 31, 30), [(4, False)], 48, (3, 3, 3), (1, 1, 1), (1, 1, 1), "simt"),
    (2, (5, 6, 7), [(4, True), (8, False)], 8, (3, 3, 3), (2, 2, 2), (1, 1, 1), "simt"),
    (1, (8, 8, 8), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (2, (9, 10, 11), [(32, True)], 64, (3, 3, 3), (2, 2, 2), (1, 1, 1), "fp32"),
    (2, (6, 6, 6), [(32, False), (32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (4, 5, 6), [(64, True)], 128, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (2, (4, 4, 4), [(128, True), (128, False)], 320, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (3, (6, 8, 10), [(64, True)], 256, (1, 1, 1), (1, 1, 1), (0, 0, 0), "fp32"),
    (2, (8, 8, 8), [(32, True)], 64, (2, 2, 2), (2, 2, 2), (0, 0, 0), "fp32"),
    (1, (12, 12, 12), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "tf32"),
    (1, (5, 6, 7), [(64, True)], 48, (1, 3, 3), (1, 2, 2), (0, 1, 1), "fp32"),
    # brick tiling: rows wider than one tile, anisotropic strides, partial N tiles
    (1, (20, 17, 130), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (2, (16, 40, 40), [(32, True)], 64, (3, 3, 3), (1, 2, 2), (1, 1, 1), "tf32"),
    (1, (7, 9, 11), [(96, True)], 96, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (9, 9, 9), [(32, True), (64, False)], 16, (3, 3, 3), (2, 1, 2), (1, 1, 1), "fp32"),
    # halo mode (unit stride, 8x16 bricks, one plane box per kz feeds the kx/ky taps)
    (2, (10, 12, 16), [(32, True), (32, False)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (9, 20, 24), [(64, True)], 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (5, 16, 16), [(32, True)], 32, (1, 3, 3), (1, 1, 1), (0, 1, 1), "fp32"),
    (1, (6, 16, 8), [(32, True)], 32, (3, 1, 1), (1, 1, 1), (1, 0, 0), "tf32"),
    (2, (7, 19, 13), [(64, True)], 48, (3, 3, 3), (1, 1, 1), (1, 1, 1), "tf32"),
    # z-streaming (fp16 pairs, 3x3x3 s1 p1, <= 32 output channels): partial bricks, 1-plane and short
    # columns, 16 output channels, 2 and 3 chunks of streamed weights, several samples
    (2, (5, 9, 17), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (1, 8, 8), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (3, 8, 8), [(32, True), (32, False)], 16, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (3, (4, 16, 8), [(96, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (40, 24, 24), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    # z-streaming schedule on 148 SMs: exactly one round of whole columns (4 x 37 columns), and two rounds
    # followed by 4 columns split into runs (2 x 150 columns)
    (4, (4, 16, 296), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (2, (9, 32, 600), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    # split TF32 (the range fallback of the default fp16-pair mode): halo, box, 128-column and concat shapes
    (2, (10, 12, 16), [(32, True), (32, False)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32-tf32x2"),
    (2, (9, 10, 11), [(32, True)], 64, (3, 3, 3), (2, 2, 2), (1, 1, 1), "fp32-tf32x2"),
    (1, (4, 5, 6), [(64, True)], 128, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32-tf32x2"),
    (1, (9, 20, 24), [(64, True)], 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32-tf32x2"),
]

PRECISION_CODES = {"fp32": 0, "tf32": 1, "simt": 2, "fp32-tf32x2": 3}


@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: f"{c[7]}-cin{[s[0] for s in c[2]]}-co{c[3]}-s{c[5][0]}")
def test_conv3d_matches_float32_reference(cuda_device, case):
    from nnunet_mlx_b200 import _native, kernels

    batch, dims, segs, cout, kernel, stride, pad, precision = case
    rng = np.random.default_rng(hash(str(case)) % 2**32)
    lazies, refs = [], []
    for channels, lazy in segs:
        lz, raw, sc, sh = _make_segment(rng, batch, dims, channels, lazy, cuda_device)
        lazies.append(lz)
        refs.append(_lazy_ref(raw, sc, sh, lazy))
    cin = sum(c for c, _ in segs)
    w = torch.from_numpy((rng.standard_normal((cout, *kernel, cin)) / np.sqrt(cin * np.prod(kernel))).astype(np.float32))
    prec = PRECISION_CODES[precision]
    wd = w.to(cuda_device)
    packed = kernels.pack_weights(wd, prec)
    if precision != "simt" and cin % 32 == 0:
        assert packed is not None, "expected the tensor-core path for this shape"
    out, partials = kernels.conv3d(lazies, wd, kernel=kernel, stride=stride, pad=pad, cout=cout, packed=packed,
                                   precision=prec)
    ref = _conv_ref(refs, w, stride, pad)
    tol = TF32_TOL if precision == "tf32" else FP32_TOL
    got = out.cpu()
    scale = ref.abs().max().item()
    np.testing.assert_allclose(got.numpy(), ref.numpy(), rtol=tol["rtol"], atol=tol["atol"] * max(1.0, scale))
    # instance-norm statistics from the per-tile partials
    sc, sh = kernels.instance_norm_finalize(partials, None, None, 1e-5)
    r = ref.double()
    mean = r.mean(dim=(1, 2, 3))
    var = r.var(dim=(1, 2, 3), unbiased=False)
    ref_scale = 1 / torch.sqrt(var + 1e-5)
    ref_shift = -mean * ref_scale
    np.testing.assert_allclose(sc.cpu().numpy(), ref_scale.numpy(), rtol=5e-3 if precision == "tf32" else 1e-4)
    np.testing.assert_allclose(sh.cpu().numpy(), ref_shift.numpy(), rtol=5e-3 if precision == "tf32" else 1e-4,
                               atol=5e-3 if precision == "tf32" else 1e-4)


def test_instance_norm_finalize_with_affine_matches_torch(cuda_device):
    from nnunet_mlx_b200 import _native, kernels
    from nnunet_mlx_b200.kernels import Lazy

    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((2, 9, 10, 11, 4)).astype(np.float32) * 3 + 7)
    w = torch.from_numpy(rng.standard_normal((4, 1, 1, 1, 4)).astype(np.float32))
    gamma = torch.from_numpy(rng.uniform(0.5, 2, 4).astype(np.float32))
    beta = torch.from_numpy(rng.standard_normal(4).astype(np.float32))
    out, partials = kernels.conv3d([Lazy(x.to(cuda_device))], w.to(cuda_device), kernel=(1, 1, 1), stride=(1, 1, 1),
                                   pad=(0, 0, 0), cout=4, precision=_native.PREC_SIMT)
    sc, sh = kernels.instance_norm_finalize(partials, gamma.to(cuda_device), beta.to(cuda_device), 1e-5)
    y = out.cpu()
    normed = y * sc.cpu()[:, None, None, None, :] + sh.cpu()[:, None, None, None, :]
    ref = F.instance_norm(y.permute(0, 4, 1, 2, 3), weight=gamma, bias=beta, eps=1e-5).permute(0, 2, 3, 4, 1)
    np.testing.assert_allclose(normed.numpy(), ref.numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("kernel,cin,cout,precision", [
    ((2, 2, 2), 16, 8, "simt"),
    ((1, 2, 2), 16, 8, "simt"),
    ((2, 2, 2), 64, 32, "fp32"),
    ((2, 2, 2), 320, 320, "fp32"),
    ((1, 2, 2), 32, 64, "fp32"),
    ((2, 2, 2), 128, 64, "tf32"),
    ((2, 2, 2), 64, 32, "fp32-tf32x2"),
])
def test_conv_transpose_matches_torch(cuda_device, kernel, cin, cout, precision):
    from nnunet_mlx_b200 import _native, kernels

    rng = np.random.default_rng(5)
    lz, raw, sc, sh = _make_segment(rng, 2, (3, 4, 5), cin, True, cuda_device)
    w = torch.from_numpy((rng.standard_normal((cout, *kernel, cin)) / np.sqrt(cin)).astype(np.float32))
    b = torch.from_numpy(rng.standard_normal(cout).astype(np.float32))
    prec = PRECISION_CODES[precision]
    wd = w.to(cuda_device)
    packed = kernels.pack_transposed_weights(wd, prec)
    if precision != "simt":
        assert packed is not None
    out = kernels.conv_transpose3d(lz, wd, b.to(cuda_device), kernel, packed=packed, precision=prec)
    x = _lazy_ref(raw, sc, sh, True).permute(0, 4, 1, 2, 3)
    ref = F.conv_transpose3d(x.double(), w.permute(4, 0, 1, 2, 3).double(), b.double(),
                             stride=kernel).permute(0, 2, 3, 4, 1).float()
    tol = TF32_TOL if precision == "tf32" else dict(rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), **tol)


@pytest.mark.parametrize("channels", [8, 6])  # float4 path; element path for a count that is not a multiple of 4
def test_residual_join_matches_reference(cuda_device, channels):
    from nnunet_mlx_b200 import kernels

    rng = np.random.default_rng(6)
    a, ra, sa, ha = _make_segment(rng, 2, (3, 4, 5), channels, True, cuda_device)
    b, rb, sb, hb = _make_segment(rng, 2, (3, 4, 5), channels, False, cuda_device)
    # branch without LeakyReLU (conv2 + norm), skip identity
    a = kernels.Lazy(a.raw, a.scale, a.shift, leaky=False)
    out = kernels.residual_join(a, b, 0.01)
    ref = F.leaky_relu(_lazy_ref(ra, sa, ha, False) + rb, 0.01)
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=1e-6)


def test_gather_views_flips(cuda_device):
    from nnunet_mlx_b200 import kernels
    from nnunet_mlx_b200.prediction.sliding_window import mirror_masks

    rng = np.random.default_rng(8)
    vol = rng.standard_normal((2, 9, 10, 11)).astype(np.float32)
    masks = mirror_masks((0, 1, 2))
    out = kernels.gather_views(torch.from_numpy(vol).to(cuda_device), (1, 2, 3), (4, 5, 6), masks).cpu().numpy()
    tile = np.moveaxis(vol[:, 1:5, 2:7, 3:9], 0, -1)
    for v, m in enumerate(masks):
        axes = tuple(a for a in range(3) if m >> a & 1)
        np.testing.assert_array_equal(out[v], np.flip(tile, axis=axes) if axes else tile)


@pytest.mark.parametrize("classes,features,axes", [(3, 32, (0, 1, 2)), (5, 16, (1, 2)), (2, 8, ())])
def test_accumulate_tile_matches_oracle_semantics(cuda_device, classes, features, axes):
    from nnunet_mlx_b200 import kernels
    from nnunet_mlx_b200.prediction.sliding_window import gaussian_importance, mirror_masks

    rng = np.random.default_rng(9)
    patch = (4, 6, 8)
    masks = mirror_masks(axes)
    views = len(masks)
    lz, raw, sc, sh = _make_segment(rng, views, patch, features, True, cuda_device)
    wseg = rng.standard_normal((classes, features)).astype(np.float32)
    bseg = rng.standard_normal(classes).astype(np.float32)
    acc0 = rng.standard_normal((7, 9, 12, classes)).astype(np.float32)
    nrm0 = rng.uniform(0.5, 1.0, (7, 9, 12)).astype(np.float32)
    acc = torch.from_numpy(acc0.copy()).to(cuda_device)
    nrm = torch.from_numpy(nrm0.copy()).to(cuda_device)
    g = gaussian_importance(patch)
    off = (2, 1, 3)
    kernels.accumulate_tile(lz, masks, torch.from_numpy(wseg).to(cuda_device), torch.from_numpy(bseg).to(cuda_device),
                            torch.from_numpy(np.ascontiguousarray(g)).to(cuda_device), acc, nrm, off, True, 0.01)
    z = _lazy_ref(raw, sc, sh, True).numpy()
    logits = z @ wseg.T + bseg  # (views, *patch, C)
    pred = logits[0].copy()
    for v in range(1, views):
        ax = tuple(a for a in range(3) if masks[v] >> a & 1)
        pred = pred + np.flip(logits[v], axis=ax)
    pred = pred / np.float32(views)
    sl = tuple(slice(o, o + p) for o, p in zip(off, patch))
    exp_acc = acc0.copy()
    exp_acc[sl] += pred * g[..., None]
    exp_nrm = nrm0.copy()
    exp_nrm[sl] += g
    np.testing.assert_allclose(acc.cpu().numpy(), exp_acc, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(nrm.cpu().numpy(), exp_nrm, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("label_dtype", [torch.uint8, torch.uint16])
def test_normalize_labels_matches_oracle(cuda_device, label_dtype):
    from oracle.sliding_window import normalized_labels

    from nnunet_mlx_b200 import kernels

    rng = np.random.default_rng(10)
    acc = rng.standard_normal((6, 7, 8, 4)).astype(np.float32)
    acc[0, 0, 0] = [1, 1, 0, 0]  # tie -> first
    nrm = rng.uniform(0.1, 2, (6, 7, 8)).astype(np.float32)
    logits, labels, invalid = kernels.normalize_labels(
        torch.from_numpy(acc).to(cuda_device), torch.from_numpy(nrm).to(cuda_device), (1, 0, 2), (4, 7, 5),
        fold_divisor=3.0, label_dtype=label_dtype)
    q = (acc / nrm[..., None]) / np.float32(3.0)
    crop = q[1:5, 0:7, 2:7]
    np.testing.assert_allclose(logits.cpu().numpy(), np.moveaxis(crop, -1, 0), rtol=1e-6, atol=1e-7)
    ref = normalized_labels(acc[1:5, 0:7, 2:7], nrm[1:5, 0:7, 2:7, None])
    got = labels.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(got, ref.astype(np.int64))
    assert int(invalid.item()) == 0


def test_normalize_labels_flags_invalid(cuda_device):
    from nnunet_mlx_b200 import kernels

    acc = torch.ones((2, 2, 2, 3), device=cuda_device)
    nrm = torch.ones((2, 2, 2), device=cuda_device)
    nrm[0, 0, 0] = 0.0
    acc[1, 1, 1, 2] = float("nan")
    _, labels, invalid = kernels.normalize_labels(acc, nrm, (0, 0, 0), (2, 2, 2), label_dtype=torch.uint8)
    assert int(invalid.item()) == 2
    lab = labels.cpu().numpy()
    assert lab[0, 0, 0] == 255 and lab[1, 1, 1] == 255 and lab[0, 1, 0] == 0


def test_c_abi_rejects_bad_arguments(cuda_device):
    from nnunet_mlx_b200 import kernels
    from nnunet_mlx_b200.errors import ContractError

    vol = torch.zeros((1, 4, 4, 4), device=cuda_device)
    with pytest.raises(ContractError, match="outside"):
        kernels.gather_views(vol, (1, 0, 0), (4, 4, 4), [0])
    x = kernels.Lazy(torch.zeros((1, 4, 4, 4, 8), device=cuda_device))
    w = torch.zeros((8, 3, 3, 3, 8), device=cuda_device)
    with pytest.raises(ContractError):
        kernels.conv3d([x], w, kernel=(3, 3, 3), stride=(1, 1, 1), pad=(1, 1, 1), cout=8, precision=7)


@pytest.mark.parametrize("cin,cout,lazy", [(32, 3, True), (4, 2, False), (64, 8, True)])
def test_pointwise_head_matches_reference(cuda_device, cin, cout, lazy):
    """1x1x1 head without statistics (the network's tile-callable seam) on the pointwise kernel."""
    from nnunet_mlx_b200 import _native, kernels

    rng = np.random.default_rng(cin + cout)
    lz, raw, sc, sh = _make_segment(rng, 2, (5, 6, 7), cin, lazy, cuda_device)
    w = torch.from_numpy(rng.standard_normal((cout, 1, 1, 1, cin)).astype(np.float32))
    b = torch.from_numpy(rng.standard_normal(cout).astype(np.float32))
    out, partials = kernels.conv3d([lz], w.to(cuda_device), kernel=(1, 1, 1), stride=(1, 1, 1), pad=(0, 0, 0),
                                   cout=cout, bias=b.to(cuda_device), precision=_native.PREC_SIMT, stats=False)
    assert partials is None
    ref = _conv_ref([_lazy_ref(raw, sc, sh, lazy)], w, (1, 1, 1), (0, 0, 0), bias=b)
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("cin,cout,stride", [(32, 32, 1), (64, 128, 1), (32, 64, 2)])
def test_fp16_pair_column_scales_cover_weight_magnitudes(cuda_device, cin, cout, stride):
    """Per-column power-of-two weight scales: columns from 1e-9 to 1e4 keep float32-level accuracy."""
    from nnunet_mlx_b200 import _native, kernels
    from nnunet_mlx_b200.kernels import Lazy

    rng = np.random.default_rng(cin + cout + stride)
    x = torch.from_numpy(rng.standard_normal((1, 8, 16, 16, cin)).astype(np.float32))
    w = rng.standard_normal((cout, 3, 3, 3, cin)) / np.sqrt(27 * cin)
    w *= 10.0 ** rng.uniform(-9, 4, (cout, 1, 1, 1, 1))
    w = torch.from_numpy(w.astype(np.float32))
    packed = kernels.pack_weights(w.to(cuda_device), _native.PREC_FP32)
    out, _ = kernels.conv3d([Lazy(x.to(cuda_device))], w.to(cuda_device), kernel=(3, 3, 3), stride=(stride,) * 3,
                            pad=(1, 1, 1), cout=cout, packed=packed, precision=_native.PREC_FP32)
    ref = _conv_ref([x], w, (stride,) * 3, (1, 1, 1)).numpy()
    got = out.cpu().numpy()
    col_scale = np.abs(ref).reshape(-1, cout).max(axis=0)
    err = np.abs(got - ref).reshape(-1, cout).max(axis=0)
    assert (err <= 2e-5 * col_scale).all(), (err / col_scale).max()


def test_fp16_pair_operand_format_and_range_events(cuda_device):
    """Prepared fp16-pair operand: hi + lo reproduces the activation to ~2^-22; |x| >= 65504 is counted."""
    from nnunet_mlx_b200 import _native, kernels
    from nnunet_mlx_b200.kernels import Lazy

    rng = np.random.default_rng(31)
    raw = rng.standard_normal((2, 3, 4, 5, 64)).astype(np.float32) * 50
    raw[0, 0, 0, 0, :5] = [65503.0, 65504.0, -70000.0, 1e9, -65504.0]  # four counted (|x| >= 65504)
    raw[1, 2, 3, 4, 7] = 3e-7                                            # subnormal hi, still reproduced
    lazy = Lazy(torch.from_numpy(raw).to(cuda_device))
    kernels.operand_range_events(reset=True)
    prepared = kernels.prepare_operand(lazy, _native.PREC_FP32, 0.01)
    assert kernels.operand_range_events(reset=True) == 4
    halves = prepared.raw.view(torch.float16).cpu().numpy().astype(np.float64)
    pairs = halves.reshape(*raw.shape[:-1], raw.shape[-1] // 32, 2, 32)
    finite = np.abs(raw) < 65504
    recon = (pairs[..., 0, :] + pairs[..., 1, :]).reshape(raw.shape)
    err = np.abs(recon[finite] - raw.astype(np.float64)[finite])
    assert (err <= 2.0 ** -21 * np.abs(raw[finite]) + 2.0 ** -25).all(), err.max()


@pytest.mark.parametrize("prepared_first", [False, True])
def test_zstream_mixes_raw_and_prepared_segments(cuda_device, prepared_first):
    """A concat whose one segment already has a prepared operand: that segment is read prepared, the other raw."""
    from nnunet_mlx_b200 import _native, kernels

    rng = np.random.default_rng(41 + prepared_first)
    dims = (6, 12, 20)
    a, ra, sa, ha = _make_segment(rng, 2, dims, 32, True, cuda_device)
    b, rb, sb, hb = _make_segment(rng, 2, dims, 32, True, cuda_device)
    kernels.prepare_operand(a if prepared_first else b, _native.PREC_FP32, 0.01)  # cached on the activation
    w = torch.from_numpy((rng.standard_normal((32, 3, 3, 3, 64)) / np.sqrt(27 * 64)).astype(np.float32))
    packed = kernels.pack_weights(w.to(cuda_device), _native.PREC_FP32)
    out, _ = kernels.conv3d([a, b], w.to(cuda_device), kernel=(3, 3, 3), stride=(1, 1, 1), pad=(1, 1, 1), cout=32,
                            packed=packed, precision=_native.PREC_FP32)
    ref = _conv_ref([_lazy_ref(ra, sa, ha, True), _lazy_ref(rb, sb, hb, True)], w, (1, 1, 1), (1, 1, 1))
    scale = ref.abs().max().item()
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=FP32_TOL["rtol"], atol=FP32_TOL["atol"] * scale)


def test_to_host_returns_fresh_arrays(cuda_device):
    """Results cross to the host through one cached page-locked buffer; each call returns its own array."""
    from nnunet_mlx_b200 import kernels

    a = torch.randn((3, 17, 33, 21), device=cuda_device)
    b = torch.randint(0, 5, (40, 50), dtype=torch.uint8, device=cuda_device)
    ha = kernels.to_host(a)
    hb = kernels.to_host(b)
    a.mul_(2)
    ha2 = kernels.to_host(a)
    np.testing.assert_array_equal(ha * 2, ha2)  # the first result was not overwritten by the second copy
    np.testing.assert_array_equal(hb, b.cpu().numpy())
    assert ha.dtype == np.float32 and hb.dtype == np.uint8 and ha.shape == (3, 17, 33, 21)


def test_conv_transpose_operand_output_decodes_to_the_float32_output(cuda_device):
    """The operand the fp32-mode transposed conv writes equals (hi + lo) its float32 result; overflow counts."""
    from nnunet_mlx_b200 import _native, kernels

    rng = np.random.default_rng(51)
    lz, raw, sc, sh = _make_segment(rng, 2, (5, 6, 7), 64, True, cuda_device)
    w = torch.from_numpy((rng.standard_normal((64, 2, 2, 2, 64)) / 8).astype(np.float32)).to(cuda_device)
    b = torch.from_numpy(rng.standard_normal(64).astype(np.float32)).to(cuda_device)
    packed = kernels.pack_transposed_weights(w, _native.PREC_FP32)
    ref = kernels.conv_transpose3d(lz, w, b, (2, 2, 2), packed=packed, precision=_native.PREC_FP32)
    kernels.operand_range_events(reset=True)
    up = kernels.conv_transpose3d_operand(lz, w, b, (2, 2, 2), packed=packed, precision=_native.PREC_FP32)
    assert isinstance(up, kernels.OperandOnly)
    assert kernels.operand_range_events(reset=True) == 0
    halves = up.raw.view(torch.float16).cpu().numpy().astype(np.float64)
    pairs = halves.reshape(*ref.shape[:-1], 2, 2, 32)  # (..., group, hi/lo, 32)
    decoded = (pairs[..., 0, :] + pairs[..., 1, :]).reshape(ref.shape)
    r = ref.cpu().numpy().astype(np.float64)
    assert (np.abs(decoded - r) <= 2.0 ** -21 * np.abs(r) + 2.0 ** -24).all()
    with pytest.raises(Exception):
        up.segment()  # not a float32 activation
    big = kernels.conv_transpose3d_operand(lz, w * 1e6, b, (2, 2, 2),
                                           packed=kernels.pack_transposed_weights(w * 1e6, _native.PREC_FP32),
                                           precision=_native.PREC_FP32)
    assert big is not None and kernels.operand_range_events(reset=True) > 0
