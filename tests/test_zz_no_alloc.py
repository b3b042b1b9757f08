"""nnb_conv3d_norm_static: the no-allocation convolution + instance-norm statistics.

Collected last on purpose (file name): the entry point's scratch is a fixed
device array shared by every call on a device, so this file also checks that
it works after the rest of the suite has run, and alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

# (batch, in_dims, segments [(channels, lazy)], cout, kernel, stride, pad, precision)
CASES = [
    (2, (12, 12, 12), [(32, True)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "fp32"),
    (1, (9, 10, 11), [(32, True), (32, False)], 64, (3, 3, 3), (2, 2, 2), (1, 1, 1), "fp32"),
    (2, (7, 8, 9), [(1, False)], 32, (3, 3, 3), (1, 1, 1), (1, 1, 1), "simt"),
]


def _segment(rng, batch, dims, channels, lazy, device):
    from nnunet_mlx_b200.kernels import Lazy

    raw = torch.from_numpy(rng.standard_normal((batch, *dims, channels)).astype(np.float32)).to(device)
    if not lazy:
        return Lazy(raw)
    scale = torch.from_numpy(rng.uniform(0.5, 1.5, (batch, channels)).astype(np.float32)).to(device)
    shift = torch.from_numpy(rng.standard_normal((batch, channels)).astype(np.float32)).to(device)
    return Lazy(raw, scale, shift, leaky=True)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[7]}-cin{sum(s[0] for s in c[2])}-co{c[3]}")
def test_static_scratch_matches_allocating_path_twice(cuda_device, case):
    from nnunet_mlx_b200 import _native, kernels

    batch, dims, segs, cout, kernel, stride, pad, precision = case
    rng = np.random.default_rng(17)
    inputs = [_segment(rng, batch, dims, c, lazy, cuda_device) for c, lazy in segs]
    cin = sum(c for c, _ in segs)
    weight = torch.from_numpy((rng.standard_normal((cout, *kernel, cin)) / np.sqrt(cin * np.prod(kernel)))
                              .astype(np.float32)).to(cuda_device)
    gamma = torch.from_numpy(rng.uniform(0.5, 1.5, cout).astype(np.float32)).to(cuda_device)
    beta = torch.from_numpy(rng.standard_normal(cout).astype(np.float32)).to(cuda_device)
    prec = {"fp32": _native.PREC_FP32, "simt": _native.PREC_SIMT}[precision]
    packed = kernels.pack_weights(weight, prec)
    geometry = dict(kernel=kernel, stride=stride, pad=pad, cout=cout, packed=packed, precision=prec)

    ref_out, partials = kernels.conv3d(inputs, weight, **geometry)
    ref_scale, ref_shift = kernels.instance_norm_finalize(partials, gamma, beta, 1e-5)
    for _ in range(2):  # two calls in a row reuse the same scratch
        out, scale, shift = kernels.conv3d_norm_static(inputs, weight, gamma=gamma, beta=beta, eps=1e-5,
                                                       **geometry)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref_out.cpu().numpy(), rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(scale.cpu().numpy(), ref_scale.cpu().numpy(), rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(shift.cpu().numpy(), ref_shift.cpu().numpy(), rtol=1e-6, atol=1e-6)


def test_static_scratch_rejects_oversized_requests():
    """Host-side size check: nothing is launched, so this runs without a GPU."""
    import ctypes

    from nnunet_mlx_b200 import _native

    lib = _native.load()
    args = _native.Conv3dArgs()
    args.batch = 8
    args.in_dims = _native.dims3((128, 128, 128))
    args.out_dims = _native.dims3((128, 128, 128))
    args.kernel = _native.dims3((3, 3, 3))
    args.stride = _native.dims3((1, 1, 1))
    args.pad = _native.dims3((1, 1, 1))
    args.num_segments = 1
    args.seg[0] = _native.Segment(256, 0, 0, 32, 0)  # never dereferenced: rejected before any launch
    args.cout = 32
    args.weight = 256
    args.out = 256
    args.partials = 0
    args.precision = _native.PREC_SIMT
    args.operand_format = 0
    status = lib.nnb_conv3d_norm_static(ctypes.byref(args), None, None, 1e-5, 256, 256, None)
    assert status == -2  # NNB_E_UNSUPPORTED
    message = lib.nnb_last_error().decode()
    assert "static scratch holds 4194304" in message
    # a caller-provided partials buffer is refused as well
    args.partials = 256
    assert lib.nnb_conv3d_norm_static(ctypes.byref(args), None, None, 1e-5, 256, 256, None) == -1
