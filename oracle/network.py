"""PyTorch-CPU float32 restatement of the reference U-Net forward -- TEST INFRASTRUCTURE.

Follows reference ``src/nnunet_mlx/model/network.py``:

* ``ConvNorm._conv_norm`` (214-237): convolution with padding ``k // 2``, then
  instance norm of ``conv + bias`` (biased variance, eps from the spec,
  ``kernels/metal_native_norm.py:92-168``), then LeakyReLU for ``ConvNormAct``;
* ``StackedConvs`` (358-410): stride on the first block only;
* ``PlainConvUNet.__call__`` (453-464) and ``_decode`` (837-877): skips popped
  deepest first, ``up{i}`` -> ``_match_spatial`` -> concat ``(up, skip)`` ->
  ``dec{i}``, segmentation head of the last decoder stage only;
* ``NonOverlappingConvTranspose3d`` (101-174): stride == kernel transposed conv
  plus bias;
* ``ResidualBlock`` (467-516), ``BottleneckResidualBlock`` (519-573),
  ``_build_residual_skip`` (576-602), ``ResidualEncoderUNet`` (655-732).

Weights are the converted checkpoint layout of reference
``storage/weights.py:32-45``: convolution ``(C_out, kD, kH, kW, C_in)`` and
transposed convolution ``(C_out, kD, kH, kW, C_in)``.  Activations inside this
oracle are torch channels-first ``(B, C, D, H, W)``; the public functions take
and return the reference's channels-last ``(B, D, H, W, C)``.

Only tests, ``smoke()`` and the bench CPU baseline may use this module.
"""

from __future__ import annotations

from collections.abc import Mapping

import numpy as np
import torch
import torch.nn.functional as F

Weights = Mapping[str, np.ndarray]


def _t(weights: Weights, key: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(weights[key], dtype=np.float32))


def _conv_weight(weights: Weights, key: str) -> torch.Tensor:
    # (C_out, k..., C_in) -> torch (C_out, C_in, k...)
    w = _t(weights, key)
    return w.permute(0, w.ndim - 1, *range(1, w.ndim - 1)).contiguous()


def _transposed_weight(weights: Weights, key: str) -> torch.Tensor:
    # (C_out, k..., C_in) -> torch ConvTranspose (C_in, C_out, k...)
    w = _t(weights, key)
    return w.permute(w.ndim - 1, 0, *range(1, w.ndim - 1)).contiguous()


def _conv(x: torch.Tensor, weights: Weights, prefix: str, stride, *, bias: bool) -> torch.Tensor:
    w = _conv_weight(weights, f"{prefix}.weight")
    kernel = tuple(w.shape[2:])
    padding = tuple(k // 2 for k in kernel)
    b = _t(weights, f"{prefix}.bias") if bias and f"{prefix}.bias" in weights else None
    op = F.conv3d if x.ndim == 5 else F.conv2d
    return op(x, w, b, stride=tuple(stride), padding=padding)


def _norm(x: torch.Tensor, weights: Weights, prefix: str, spec) -> torch.Tensor:
    gamma = _t(weights, f"{prefix}.weight") if spec.norm_affine else None
    beta = _t(weights, f"{prefix}.bias") if spec.norm_affine else None
    return F.instance_norm(x, weight=gamma, bias=beta, eps=spec.norm_eps)


def conv_norm(x, weights, prefix, stride, spec, *, act: bool, conv_bias: bool | None = None):
    """``ConvNorm`` / ``ConvNormAct`` (reference network.py:177-355)."""
    use_bias = spec.conv_bias if conv_bias is None else conv_bias
    y = _norm(_conv(x, weights, f"{prefix}.conv", stride, bias=use_bias), weights, f"{prefix}.norm", spec)
    return F.leaky_relu(y, spec.leaky_slope) if act else y


def _match_spatial(values: torch.Tensor, reference: torch.Tensor) -> torch.Tensor:
    """Centre crop / zero pad (reference network.py:898-916)."""
    for axis in range(2, values.ndim):
        delta = int(values.shape[axis] - reference.shape[axis])
        if delta > 0:
            start = delta // 2
            values = values.narrow(axis, start, int(reference.shape[axis]))
        elif delta < 0:
            before = (-delta) // 2
            after = -delta - before
            pad = [0, 0] * (values.ndim - 2)
            # F.pad order: last axis first
            index = (values.ndim - 1 - axis) * 2
            pad[index], pad[index + 1] = before, after
            values = F.pad(values, pad)
    return values


def _decode(x_skips: list[torch.Tensor], weights: Weights, spec) -> torch.Tensor:
    skips = list(x_skips)
    hidden = skips.pop()
    decoders = len(spec.features) - 1
    for index in range(decoders):
        source = len(spec.features) - 1 - index
        stride = tuple(spec.strides[source])
        skip = skips.pop()
        w = _transposed_weight(weights, f"up{index}.weight")
        b = _t(weights, f"up{index}.bias") if f"up{index}.bias" in weights else None
        op = F.conv_transpose3d if hidden.ndim == 5 else F.conv_transpose2d
        up = op(hidden, w, b, stride=stride)
        hidden = torch.cat((_match_spatial(up, skip), skip), dim=1)
        for block in range(spec.decoder_convs[index]):
            hidden = conv_norm(hidden, weights, f"dec{index}.block{block}", (1,) * len(stride), spec, act=True)
    last = decoders - 1
    return _conv(hidden, weights, f"seg{last}", (1,) * (hidden.ndim - 2), bias=True)


def plain_forward_cf(x: torch.Tensor, weights: Weights, spec) -> torch.Tensor:
    """PlainConvUNet forward on channels-first torch input (network.py:413-464)."""
    skips = []
    hidden = x
    for stage in range(len(spec.features)):
        for block in range(spec.encoder_convs[stage]):
            stride = spec.strides[stage] if block == 0 else (1,) * len(spec.strides[stage])
            hidden = conv_norm(hidden, weights, f"enc{stage}.block{block}", stride, spec, act=True)
        skips.append(hidden)
    return _decode(skips, weights, spec)


def _residual_block(x, weights, prefix, stride, in_ch, out_ch, spec, bottleneck: bool):
    unit = (1,) * len(stride)
    residual = x
    if tuple(stride) != unit:
        pool = F.avg_pool3d if x.ndim == 5 else F.avg_pool2d
        residual = pool(residual, kernel_size=tuple(stride), stride=tuple(stride))
    if in_ch != out_ch:
        residual = conv_norm(residual, weights, f"{prefix}.proj", unit, spec, act=False, conv_bias=False)
    if bottleneck:
        h = conv_norm(x, weights, f"{prefix}.conv1", unit, spec, act=True)
        h = conv_norm(h, weights, f"{prefix}.conv2", stride, spec, act=True)
        h = conv_norm(h, weights, f"{prefix}.conv3", unit, spec, act=False)
    else:
        h = conv_norm(x, weights, f"{prefix}.conv1", stride, spec, act=True)
        h = conv_norm(h, weights, f"{prefix}.conv2", unit, spec, act=False)
    return F.leaky_relu(h + residual, spec.leaky_slope)


def residual_forward_cf(x: torch.Tensor, weights: Weights, spec) -> torch.Tensor:
    """ResidualEncoderUNet forward on channels-first input (network.py:655-732)."""
    unit = (1,) * len(spec.strides[0])
    hidden = conv_norm(x, weights, "stem", unit, spec, act=True)
    in_ch = spec.stem_channels or spec.features[0]
    skips = []
    bottleneck = getattr(spec, "bottleneck_channels", None) is not None
    for stage, out_ch in enumerate(spec.features):
        for block in range(spec.encoder_blocks[stage]):
            stride = spec.strides[stage] if block == 0 else unit
            block_in = in_ch if block == 0 else out_ch
            hidden = _residual_block(hidden, weights, f"res{stage}.block{block}", stride,
                                     block_in, out_ch, spec, bottleneck)
        skips.append(hidden)
        in_ch = out_ch
    return _decode(skips, weights, spec)


def forward(x_channels_last: np.ndarray | torch.Tensor, weights: Weights, spec) -> np.ndarray:
    """Channels-last ``(B, *spatial, C_in)`` -> channels-last ``(B, *spatial, C)`` logits."""
    x = torch.as_tensor(np.asarray(x_channels_last, dtype=np.float32))
    x = x.permute(0, x.ndim - 1, *range(1, x.ndim - 1)).contiguous()
    with torch.no_grad():
        if hasattr(spec, "encoder_blocks"):
            y = residual_forward_cf(x, weights, spec)
        else:
            y = plain_forward_cf(x, weights, spec)
    return y.permute(0, *range(2, y.ndim), 1).contiguous().numpy()


def tf32_round(t: torch.Tensor) -> torch.Tensor:
    """Round float32 values to TF32 (10 explicit mantissa bits), nearest-even.

    Used only by tests that estimate how much a TF32 tensor-core forward can
    drift from the float32 oracle.
    """
    bits = t.contiguous().view(torch.int32)
    lsb = (bits >> 13) & 1
    rounded = (bits + 0x0FFF + lsb) & ~0x1FFF
    return rounded.view(torch.float32)


def fp16_pair(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Split float32 values into the fp16-pair operand: ``hi = fp16(t)``, ``lo = fp16(t - hi)``.

    ``hi + lo`` reproduces ``t`` to ~2^-22 relative, or 2^-25 absolute where
    ``lo`` is subnormal, while ``|t| < 65504``.  Used only by tests that check
    the numerics of the default tensor-core mode.
    """
    hi = t.to(torch.float16).to(torch.float32)
    lo = (t - hi).to(torch.float16).to(torch.float32)
    return hi, lo


def fp16_pair_products(op, transposed: bool = False):
    """``op`` (a float32 convolution) recomputed with the default mode's three fp16-pair products.

    Activations split with :func:`fp16_pair`; weights scaled by a power of two
    per GEMM column (output channel, or (output channel, tap) for a stride ==
    kernel transposed convolution) so that their maximum is below 2^14, then
    split.  The result is ``conv(a_hi, w_hi) + conv(a_hi, w_lo) + conv(a_lo,
    w_hi)`` divided by the column scale, the sum the tensor cores form.  Test
    infrastructure only.
    """
    def conv(x, w, b=None, **kwargs):
        # weight layout: conv (C_out, C_in, *k); transposed conv (C_in, C_out, *k)
        reduce_dims = (0,) if transposed else tuple(range(1, w.ndim))
        m = w.abs().amax(dim=reduce_dims, keepdim=True).double().numpy()
        _, e = np.frexp(np.where(m > 0, m, 1.0))
        scale = torch.from_numpy(np.where(m > 0, np.ldexp(1.0, 14 - e), 1.0).astype(np.float32))
        a_hi, a_lo = fp16_pair(x)
        w_hi, w_lo = fp16_pair(w * scale)
        out = op(a_hi, w_hi, None, **kwargs) + (op(a_hi, w_lo, None, **kwargs) + op(a_lo, w_hi, None, **kwargs))
        channel = (1, -1) + (1,) * (x.ndim - 2)
        if transposed:
            # output position p along an axis was produced by tap p % k
            k = tuple(int(v) for v in w.shape[2:])
            inv = (1.0 / scale).reshape(w.shape[1], *k)
            out = out * inv.repeat(1, *(o // kk for o, kk in zip(out.shape[2:], k))).unsqueeze(0)
        else:
            out = out / scale.reshape(channel)
        return out if b is None else out + b.reshape(channel)
    return conv
