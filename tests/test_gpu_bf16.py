"""BF16-in / float32-accumulate tensor-core convolutions on B200 against exact references.

A bf16 x bf16 product is exact in float32, so the device result of
``precision="bf16"`` equals the float64 convolution of the bf16-rounded
activation and weights up to float32 accumulation rounding.  The reference
here rounds the same way the device does: the lazy affine is one fused
multiply-add rounded to float32, LeakyReLU in float32, then round-to-nearest-
even bf16 (``torch.bfloat16``); weights are rounded to bf16.  This checks the
operand layouts, swizzles, descriptors and MMA issue of the z-streaming,
halo and box kernels and of the transposed convolution exactly, independent
of the looser bound bf16 has against float32 (``test_gpu_benchmark_parity``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

ACC_TOL = 2e-5  # float32 accumulation of exact products, relative to the output's largest magnitude


def _act_ref(raw, scale, shift, leaky, slope=0.01):
    """The device activation: fma(raw, scale, shift) rounded once to float32, then LeakyReLU in float32."""
    if scale is None:
        y = raw
    else:
        y = (raw.double() * scale.double()[:, None, None, None, :] + shift.double()[:, None, None, None, :]).float()
        if leaky:
            y = torch.where(y >= 0, y, y * slope)
    return y.to(torch.bfloat16).double()


def _segment(rng, batch, dims, channels, lazy, device):
    from nnunet_mlx_b200.kernels import Lazy

    raw = torch.from_numpy(rng.standard_normal((batch, *dims, channels)).astype(np.float32) * 2 + 0.5)
    if not lazy:
        return Lazy(raw.to(device)), _act_ref(raw, None, None, False)
    scale = torch.from_numpy(rng.uniform(0.5, 1.5, (batch, channels)).astype(np.float32))
    shift = torch.from_numpy(rng.standard_normal((batch, channels)).astype(np.float32))
    return Lazy(raw.to(device), scale.to(device), shift.to(device), leaky=True), _act_ref(raw, scale, shift, True)


BF16_CASES = [
    # (batch, in_dims, segments [(channels, lazy)], cout, kernel, stride, pad, expected kernel)
    (2, (5, 9, 17), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (1, (40, 24, 24), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (2, (9, 32, 600), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (1, (1, 8, 8), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (3, (4, 16, 8), [(96, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (1, (3, 8, 8), [(32, True), (32, False)], 16, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_zstream_kernel"),
    (1, (9, 20, 24), [(64, True)], 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_halo_kernel"),
    (2, (10, 12, 16), [(64, True), (64, False)], 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_halo_kernel"),
    (2, (9, 10, 11), [(32, True)], 64, (3, 3, 3), (2, 2, 2), (1, 1, 1), "conv3d_tc_kernel"),
    (1, (4, 5, 6), [(64, True)], 128, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_tc_kernel"),
    (2, (4, 4, 4), [(128, True), (128, False)], 320, (3, 3, 3), (1, 1, 1), (1, 1, 1), "conv3d_tc_kernel"),
    (3, (6, 8, 10), [(64, True)], 256, (1, 1, 1), (1, 1, 1), (0, 0, 0), "conv3d_tc_kernel"),
]


@pytest.mark.parametrize("case", BF16_CASES, ids=lambda c: f"{c[7]}-cin{[s[0] for s in c[2]]}-co{c[3]}-s{c[5][0]}")
def test_bf16_conv_equals_rounded_operand_convolution(cuda_device, case):
    from nnunet_mlx_b200 import _native, kernels

    batch, dims, segs, cout, kernel, stride, pad, expected = case
    rng = np.random.default_rng(abs(hash(str(case))) % 2**32)
    lazies, refs = [], []
    for channels, lazy in segs:
        lz, ref = _segment(rng, batch, dims, channels, lazy, cuda_device)
        lazies.append(lz)
        refs.append(ref)
    cin = sum(c for c, _ in segs)
    w = torch.from_numpy((rng.standard_normal((cout, *kernel, cin)) / np.sqrt(cin * np.prod(kernel))).astype(np.float32))
    wd = w.to(cuda_device)
    packed = kernels.pack_weights(wd, _native.PREC_BF16)
    assert packed is not None
    out, partials = kernels.conv3d(lazies, wd, kernel=kernel, stride=stride, pad=pad, cout=cout, packed=packed,
                                   precision=_native.PREC_BF16)
    kernels.PROFILE.enable(True)
    try:
        kernels.conv3d(lazies, wd, kernel=kernel, stride=stride, pad=pad, cout=cout, packed=packed,
                       precision=_native.PREC_BF16)
        torch.cuda.synchronize()
        launched = kernels.PROFILE.trace()[-1]["detail"].rsplit(" ", 1)[-1]
    finally:
        kernels.PROFILE.enable(False)
        kernels.PROFILE.reset()
    assert launched == expected
    x = torch.cat(refs, dim=-1).permute(0, 4, 1, 2, 3)
    wr = w.to(torch.bfloat16).double().permute(0, 4, 1, 2, 3)
    ref = F.conv3d(x, wr, None, stride=stride, padding=pad).permute(0, 2, 3, 4, 1)
    got = out.cpu().double()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= ACC_TOL * scale, (err, scale)
    sc, sh = kernels.instance_norm_finalize(partials, None, None, 1e-5)
    var = ref.var(dim=(1, 2, 3), unbiased=False)
    np.testing.assert_allclose(sc.cpu().numpy(), (1 / torch.sqrt(var + 1e-5)).numpy(), rtol=1e-4)


def test_bf16_transposed_conv_writes_the_next_operand(cuda_device):
    """The decoder's up-convolution writes the bf16 half of its operand rows; the concat convolution reads them."""
    from nnunet_mlx_b200 import _native, kernels

    rng = np.random.default_rng(7)
    x, x_ref = _segment(rng, 2, (4, 8, 8), 64, True, cuda_device)
    w = torch.from_numpy((rng.standard_normal((32, 2, 2, 2, 64)) / 8).astype(np.float32))
    b = torch.from_numpy((0.1 * rng.standard_normal(32)).astype(np.float32))
    wd, bd = w.to(cuda_device), b.to(cuda_device)
    packed = kernels.pack_transposed_weights(wd, _native.PREC_BF16)
    up = kernels.conv_transpose3d_operand(x, wd, bd, (2, 2, 2), 0.01, packed=packed, precision=_native.PREC_BF16)
    assert isinstance(up, kernels.OperandOnly) and up.precision == _native.PREC_BF16
    rows = up.raw.cpu().view(torch.bfloat16).double()  # (B, D, H, W, 64): 32 bf16 values, then an unread half
    values = rows[..., :32]
    # the float32 transposed conv of the bf16 operands, then bf16: equal except where the float32 sum lies
    # within accumulation rounding of a bf16 rounding midpoint (then one bf16 step apart)
    up_ref = F.conv_transpose3d(x_ref.permute(0, 4, 1, 2, 3), w.to(torch.bfloat16).double().permute(4, 0, 1, 2, 3),
                                b.double(), stride=2).permute(0, 2, 3, 4, 1)
    expect = up_ref.float().to(torch.bfloat16).double()
    step = expect.abs().clamp_min(1e-30) * 2.0 ** -7
    off = (values - expect).abs()
    assert (off <= step).all()
    assert (off > 0).float().mean().item() < 1e-3
    # the concat convolution reads exactly those operand values
    skip, skip_ref = _segment(rng, 2, (8, 16, 16), 32, True, cuda_device)
    wc = torch.from_numpy((rng.standard_normal((32, 3, 3, 3, 64)) / np.sqrt(27 * 64)).astype(np.float32))
    wcd = wc.to(cuda_device)
    out, _ = kernels.conv3d([up, skip], wcd, kernel=(3, 3, 3), stride=(1, 1, 1), pad=(1, 1, 1), cout=32,
                            packed=kernels.pack_weights(wcd, _native.PREC_BF16), precision=_native.PREC_BF16)
    xin = torch.cat([values, skip_ref], dim=-1).permute(0, 4, 1, 2, 3)
    ref = F.conv3d(xin, wc.to(torch.bfloat16).double().permute(0, 4, 1, 2, 3), None, padding=1).permute(0, 2, 3, 4, 1)
    scale = ref.abs().max().item()
    assert (out.cpu().double() - ref).abs().max().item() <= ACC_TOL * scale


def test_bf16_network_runs_and_stays_close(cuda_device):
    """A mid-size network in bf16 against the float32 oracle (bound of the single-pass mode)."""
    from oracle import network as onet

    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
    from nnunet_mlx_b200.synthetic import seeded_weights

    k3 = (3, 3, 3)
    spec = PlainConvUNetSpec(input_channels=1, num_classes=3, features=(32, 64, 128), kernel_sizes=(k3,) * 3,
                             strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)), encoder_convs=(2, 2, 2), decoder_convs=(2, 2))
    weights = seeded_weights(spec, 3)
    net = build_network(spec, precision="bf16", device=cuda_device).load_weights(weights)
    x = np.random.default_rng(4).standard_normal((2, 16, 24, 16, 1)).astype(np.float32)
    got = net(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    ref = onet.forward(x, weights, spec)
    assert np.abs(got - ref).max() <= 0.5
    assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.95
