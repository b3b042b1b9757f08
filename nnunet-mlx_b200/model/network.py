"""PlainConvUNet and ResidualEncoderUNet on B200: the network forward of the inference path.

Same stage layout, parameter names and converted weight format as reference
``src/nnunet_mlx/model/network.py`` (``PlainConvUNet`` 413-464,
``ResidualEncoderUNet`` 655-732, ``_build_decoder`` 771-809, ``_decode``
837-877): ``enc{i}.block{j}`` / ``stem`` / ``res{i}.block{b}.{conv1,conv2,conv3,proj}``
convolution + instance-norm blocks, ``up{i}`` stride == kernel transposed
convolutions, ``dec{i}.block{j}`` decoder blocks over ``concat(up, skip)`` and
``seg{i}`` heads of which only the last runs.

Execution differs from the reference by design:

* every convolution is one ``nnb_conv3d`` call (tcgen05 tensor cores, or CUDA
  cores outside the tensor-core envelope) that also writes per-tile
  instance-norm partials; ``nnb_instance_norm_finalize`` turns them into a
  per-(sample, channel) affine;
* the affine + LeakyReLU is not materialised: the next consumer (convolution,
  transposed convolution, residual join or the fused segmentation head)
  applies it while loading (``kernels.Lazy``);
* the convolution bias before an instance norm is dropped (the norm removes
  any per-channel constant, reference ``ConvNorm._conv_norm`` 214-237 adds it
  only to normalise it away);
* the decoder concat is two K segments of one convolution, never materialised
  (reference ``_split_concatenated_input`` 305-322 does this for some shapes);
* a pooled residual skip ``proj(avgpool_s(x))`` (``_build_residual_skip``
  576-602) runs as one convolution with kernel = stride = s and weights
  ``W / prod(s)`` on every tap, which is the same linear map.

Inputs are batches of channels-last tiles ``(B, D, H, W, C_in)``; the
sliding-window predictor passes the mirrored views of a tile as the batch.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, replace

import numpy as np
import torch

from nnunet_mlx_b200 import _native, kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.kernels import Lazy
from nnunet_mlx_b200.model.topology import NetworkSpec, PlainConvUNetSpec, ResidualEncoderUNetSpec
from nnunet_mlx_b200.storage.weights import validate_weights

PRECISIONS = {"fp32": _native.PREC_FP32, "tf32": _native.PREC_TF32, "simt": _native.PREC_SIMT,
              "fp32-tf32x2": _native.PREC_FP32_TF32, "bf16": _native.PREC_BF16}
# "fp32" runs split fp16 pairs, exact to float32 level while every activation stays below 65504 in
# magnitude; a forward that met a larger one is recomputed in split TF32 (see range_fallback).
RANGE_FALLBACK = {"fp32": "fp32-tf32x2"}


@dataclass
class ConvLayer:
    """One convolution (+ optional instance norm) with its device weights."""

    weight: torch.Tensor
    kernel: tuple[int, int, int]
    stride: tuple[int, int, int]
    pad: tuple[int, int, int]
    cout: int
    gamma: torch.Tensor | None
    beta: torch.Tensor | None
    bias: torch.Tensor | None = None
    packed: torch.Tensor | None = None


def _unit(spec) -> tuple[int, ...]:
    return (1,) * spec.spatial_dims


class _UNetBase:
    """Shared decoder, weight residency and execution policy."""

    spec: NetworkSpec

    def __init__(self, spec: NetworkSpec, *, precision: str = "fp32", device: str | torch.device = "cuda") -> None:
        if spec.spatial_dims != 3:
            raise ContractError("the B200 inference path implements 3-D networks")
        if precision not in PRECISIONS:
            raise ContractError(f"unknown precision {precision!r}; expected one of {sorted(PRECISIONS)}")
        self.spec = spec
        self.precision = precision
        self.device = torch.device(device)
        self.training = False
        self.layers: dict[str, ConvLayer] = {}
        self.up: dict[int, tuple[torch.Tensor, torch.Tensor | None, tuple[int, int, int], torch.Tensor | None]] = {}
        self.seg_weight: torch.Tensor | None = None
        self.seg_bias: torch.Tensor | None = None
        self._loaded = False
        self._fallback: _UNetBase | None = None

    # ------------------------------------------------------------------ weights
    def _tensor(self, array: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).to(self.device)

    def _conv_layer(self, weights, prefix: str, stride, *, conv_bias: bool, norm: bool = True,
                    weight_override: np.ndarray | None = None, pad: tuple[int, int, int] | None = None) -> None:
        w = weights[f"{prefix}.conv.weight"] if weight_override is None else weight_override
        kernel = tuple(int(k) for k in w.shape[1:-1])
        layer = ConvLayer(
            weight=self._tensor(w), kernel=kernel, stride=tuple(int(s) for s in stride),
            pad=tuple(k // 2 for k in kernel) if pad is None else pad, cout=int(w.shape[0]),
            gamma=self._tensor(weights[f"{prefix}.norm.weight"]) if norm and self.spec.norm_affine else None,
            beta=self._tensor(weights[f"{prefix}.norm.bias"]) if norm and self.spec.norm_affine else None,
        )
        del conv_bias  # a bias before instance norm cancels exactly; it is not applied
        layer.packed = kernels.pack_weights(layer.weight, PRECISIONS[self.precision])
        self.layers[prefix] = layer

    def _load_decoder(self, weights) -> None:
        spec = self.spec
        stages = len(spec.features)
        for d in range(stages - 1):
            src = stages - 1 - d
            w = self._tensor(weights[f"up{d}.weight"])
            b = weights.get(f"up{d}.bias")
            self.up[d] = (w, None if b is None else self._tensor(b), tuple(int(k) for k in spec.strides[src]),
                          kernels.pack_transposed_weights(w, PRECISIONS[self.precision]))
            for blk in range(spec.decoder_convs[d]):
                self._conv_layer(weights, f"dec{d}.block{blk}", _unit(spec), conv_bias=spec.conv_bias)
        last = stages - 2
        seg = weights[f"seg{last}.weight"]
        self.seg_weight = self._tensor(seg.reshape(seg.shape[0], seg.shape[-1]))
        self.seg_bias = self._tensor(weights[f"seg{last}.bias"])

    def load_weights(self, weights) -> "_UNetBase":
        """Strictly validate converted weights (reference ``load_converted_state``) and upload them."""
        checked = validate_weights(self.spec, weights)
        self.layers = {}
        self.up = {}
        self._fallback = None
        self._load(checked)
        self._load_decoder(checked)
        self._loaded = True
        return self

    @property
    def range_guarded(self) -> bool:
        """True when this network's tensor-core operands have a bounded range (split fp16 pairs)."""
        return self.precision in RANGE_FALLBACK

    def range_fallback(self) -> "_UNetBase":
        """This network computing in split TF32 (same device weights, own weight images, built once).

        Used to recompute a volume in which an activation exceeded the fp16-pair
        operand range (``kernels.operand_range_events``).
        """
        target = RANGE_FALLBACK.get(self.precision)
        if target is None:
            return self
        if self._fallback is None:
            if not self._loaded:
                raise ContractError("network weights are not loaded")
            prec = PRECISIONS[target]
            twin = copy.copy(self)
            twin.precision = target
            twin._fallback = None
            twin.layers = {name: replace(layer, packed=kernels.pack_weights(layer.weight, prec))
                           for name, layer in self.layers.items()}
            twin.up = {d: (w, b, k, kernels.pack_transposed_weights(w, prec)) for d, (w, b, k, _) in self.up.items()}
            self._fallback = twin
        return self._fallback

    def _load(self, weights) -> None:  # encoder, per subclass
        raise NotImplementedError

    # ------------------------------------------------------------------ execution
    def _conv_norm(self, prefix: str, inputs: list[Lazy], *, act: bool) -> Lazy:
        layer = self.layers[prefix]
        out, partials = kernels.conv3d(
            inputs, layer.weight, kernel=layer.kernel, stride=layer.stride, pad=layer.pad, cout=layer.cout,
            packed=layer.packed, precision=PRECISIONS[self.precision], slope=self.spec.leaky_slope)
        scale, shift = kernels.instance_norm_finalize(partials, layer.gamma, layer.beta, self.spec.norm_eps)
        return Lazy(out, scale, shift, leaky=act)

    def _decode(self, skips: list[Lazy]) -> Lazy:
        spec = self.spec
        hidden = skips.pop()
        for d in range(len(spec.features) - 1):
            weight, bias, kernel, packed = self.up[d]
            skip = skips.pop()
            up = kernels.conv_transpose3d_operand(hidden, weight, bias, kernel, spec.leaky_slope, packed=packed,
                                                  precision=PRECISIONS[self.precision])
            up = _match_spatial(up, skip)
            hidden = self._conv_norm(f"dec{d}.block0", [up, skip], act=True)
            for blk in range(1, spec.decoder_convs[d]):
                hidden = self._conv_norm(f"dec{d}.block{blk}", [hidden], act=True)
        return hidden

    def forward_features(self, x: torch.Tensor) -> Lazy:
        """Channels-last ``(B, *patch, C_in)`` -> lazy features of the last decoder stage."""
        if not self._loaded:
            raise ContractError("network weights are not loaded")
        if x.ndim != 5 or int(x.shape[-1]) != self.spec.input_channels:
            raise ContractError(f"expected (B, D, H, W, {self.spec.input_channels}) input, got {tuple(x.shape)}")
        if x.device != self.device and not (x.is_cuda and self.device.type == "cuda"):
            raise ContractError("input must be on the network's CUDA device")
        return self._forward(Lazy(x.contiguous()))

    def _forward(self, x: Lazy) -> Lazy:
        raise NotImplementedError

    def __call__(self, values: torch.Tensor) -> torch.Tensor:
        """``PredictionModel`` seam (reference ``model/types.py:14``): tile batch -> float32 logits."""
        features = self.forward_features(values)
        classes = int(self.seg_weight.shape[0])
        w = self.seg_weight.reshape(classes, 1, 1, 1, -1).contiguous()
        logits, _ = kernels.conv3d([features], w, kernel=(1, 1, 1), stride=(1, 1, 1), pad=(0, 0, 0),
                                   cout=classes, bias=self.seg_bias, precision=_native.PREC_SIMT,
                                   slope=self.spec.leaky_slope, stats=False)
        return logits

    def eval(self) -> "_UNetBase":
        return self


def _match_spatial(up: Lazy, skip: Lazy) -> Lazy:
    """Centre crop / zero pad of the up-sampled tensor (reference network.py:898-916).

    An operand-only activation is cropped / padded in its operand form (zero is
    the all-zero fp16 pair), so it stays operand-only.
    """
    if up.spatial == skip.spatial:
        return up
    raw = up.raw
    for axis in range(3):
        delta = int(raw.shape[axis + 1] - skip.spatial[axis])
        if delta > 0:
            raw = raw.narrow(axis + 1, delta // 2, skip.spatial[axis])
        elif delta < 0:
            before = (-delta) // 2
            shape = list(raw.shape)
            shape[axis + 1] = skip.spatial[axis]
            padded = torch.zeros(shape, dtype=raw.dtype, device=raw.device)
            padded.narrow(axis + 1, before, raw.shape[axis + 1]).copy_(raw)
            raw = padded
    if isinstance(up, kernels.OperandOnly):
        return kernels.OperandOnly(raw.contiguous(), up.precision)
    return Lazy(raw.contiguous())


class PlainConvUNet(_UNetBase):
    """Plan-driven ``PlainConvUNet`` (reference network.py:413-464)."""

    def __init__(self, spec: PlainConvUNetSpec, **kwargs) -> None:
        if not isinstance(spec, PlainConvUNetSpec):
            raise ContractError("PlainConvUNet requires a PlainConvUNetSpec")
        super().__init__(spec, **kwargs)

    def _load(self, weights) -> None:
        spec = self.spec
        for s in range(len(spec.features)):
            for b in range(spec.encoder_convs[s]):
                stride = spec.strides[s] if b == 0 else _unit(spec)
                self._conv_layer(weights, f"enc{s}.block{b}", stride, conv_bias=spec.conv_bias)

    def _forward(self, x: Lazy) -> Lazy:
        spec = self.spec
        skips: list[Lazy] = []
        hidden = x
        for s in range(len(spec.features)):
            for b in range(spec.encoder_convs[s]):
                hidden = self._conv_norm(f"enc{s}.block{b}", [hidden], act=True)
            skips.append(hidden)
        return self._decode(skips)


class ResidualEncoderUNet(_UNetBase):
    """Residual encoder (BasicBlockD / BottleneckD) + plain decoder (reference network.py:655-732)."""

    def __init__(self, spec: ResidualEncoderUNetSpec, **kwargs) -> None:
        if not isinstance(spec, ResidualEncoderUNetSpec):
            raise ContractError("ResidualEncoderUNet requires a ResidualEncoderUNetSpec")
        super().__init__(spec, **kwargs)
        self.skip_kind: dict[str, str] = {}

    def _load(self, weights) -> None:
        spec = self.spec
        unit = _unit(spec)
        self._conv_layer(weights, "stem", unit, conv_bias=spec.conv_bias)
        cin = spec.effective_stem_channels
        for s, f in enumerate(spec.features):
            for b in range(spec.encoder_blocks[s]):
                stride = tuple(spec.strides[s]) if b == 0 else unit
                bin_ = cin if b == 0 else f
                p = f"res{s}.block{b}"
                if spec.bottleneck_channels is None:
                    self._conv_layer(weights, f"{p}.conv1", stride, conv_bias=spec.conv_bias)
                    self._conv_layer(weights, f"{p}.conv2", unit, conv_bias=spec.conv_bias)
                else:
                    self._conv_layer(weights, f"{p}.conv1", unit, conv_bias=spec.conv_bias)
                    self._conv_layer(weights, f"{p}.conv2", stride, conv_bias=spec.conv_bias)
                    self._conv_layer(weights, f"{p}.conv3", unit, conv_bias=spec.conv_bias)
                pooled = stride != unit
                if bin_ != f:
                    w = weights[f"{p}.proj.conv.weight"]  # (f, 1, 1, 1, bin_)
                    if pooled:
                        taps = np.broadcast_to(w, (w.shape[0], *stride, w.shape[-1])) / float(np.prod(stride))
                        self._conv_layer(weights, f"{p}.proj", stride, conv_bias=False,
                                         weight_override=np.ascontiguousarray(taps, dtype=np.float32),
                                         pad=(0, 0, 0))
                    else:
                        self._conv_layer(weights, f"{p}.proj", unit, conv_bias=False)
                    self.skip_kind[p] = "proj"
                elif pooled:
                    eye = np.zeros((f, *stride, f), dtype=np.float32)
                    eye[np.arange(f), ..., np.arange(f)] = 1.0 / float(np.prod(stride))
                    self.layers[f"{p}.pool"] = ConvLayer(
                        weight=self._tensor(eye), kernel=tuple(stride), stride=tuple(stride), pad=(0, 0, 0),
                        cout=f, gamma=None, beta=None)
                    self.layers[f"{p}.pool"].packed = kernels.pack_weights(self.layers[f"{p}.pool"].weight,
                                                                           PRECISIONS[self.precision])
                    self.skip_kind[p] = "pool"
                else:
                    self.skip_kind[p] = "identity"
            cin = f

    def _block(self, p: str, x: Lazy) -> Lazy:
        spec = self.spec
        if spec.bottleneck_channels is None:
            h = self._conv_norm(f"{p}.conv1", [x], act=True)
            h = self._conv_norm(f"{p}.conv2", [h], act=False)
        else:
            h = self._conv_norm(f"{p}.conv1", [x], act=True)
            h = self._conv_norm(f"{p}.conv2", [h], act=True)
            h = self._conv_norm(f"{p}.conv3", [h], act=False)
        kind = self.skip_kind[p]
        if kind == "proj":
            skip = self._conv_norm(f"{p}.proj", [x], act=False)
        elif kind == "pool":
            layer = self.layers[f"{p}.pool"]
            pooled, _ = kernels.conv3d([x], layer.weight, kernel=layer.kernel, stride=layer.stride, pad=layer.pad,
                                       cout=layer.cout, packed=layer.packed, precision=PRECISIONS[self.precision],
                                       slope=spec.leaky_slope, stats=False)
            skip = Lazy(pooled)
        else:
            skip = x
        return Lazy(kernels.residual_join(h, skip, spec.leaky_slope))

    def _forward(self, x: Lazy) -> Lazy:
        spec = self.spec
        hidden = self._conv_norm("stem", [x], act=True)
        skips: list[Lazy] = []
        for s in range(len(spec.features)):
            for b in range(spec.encoder_blocks[s]):
                hidden = self._block(f"res{s}.block{b}", hidden)
            skips.append(hidden)
        return self._decode(skips)


def build_network(spec: NetworkSpec, **kwargs) -> _UNetBase:
    """Network class for a spec (reference ``model/factory.py:17-65``)."""
    if isinstance(spec, ResidualEncoderUNetSpec):
        return ResidualEncoderUNet(spec, **kwargs)
    return PlainConvUNet(spec, **kwargs)
