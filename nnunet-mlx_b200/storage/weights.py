"""Converted checkpoint weight format: key names, layouts and expected shapes.

The converted (MLX-layout) checkpoint is what this package reads, so that model
folders produced by the reference's converter load unchanged:

* key and layout mapping from upstream torch ``state_dict`` keys -- same
  results as reference ``src/nnunet_mlx/storage/weights.py:48-123``
  (``map_key_and_layout``) and ``126-182`` (``convert_state_dict``);
  convolution ``(C_out, C_in, *k) -> (C_out, *k, C_in)``, transposed
  convolution ``(C_in, C_out, *k) -> (C_out, *k, C_in)``;
* ``expected_shapes(spec)`` lists every parameter a network of ``spec`` owns,
  i.e. the set a strict load (reference ``load_converted_state``, 185-192)
  requires, including all segmentation heads (reference network.py:773-775).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import numpy as np

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.topology import NetworkSpec, ResidualEncoderUNetSpec


@dataclass(frozen=True, slots=True)
class ConvertedState:
    weights: dict[str, np.ndarray]
    dropped_keys: tuple[str, ...]


def _conv_layout(array: np.ndarray) -> np.ndarray:
    if array.ndim not in (4, 5):
        raise ContractError(f"expected a 2-D or 3-D convolution weight, got {array.shape}")
    return np.transpose(array, (0, *range(2, array.ndim), 1))


def _transposed_layout(array: np.ndarray) -> np.ndarray:
    if array.ndim not in (4, 5):
        raise ContractError(f"expected a 2-D or 3-D transposed weight, got {array.shape}")
    return np.transpose(array, (1, *range(2, array.ndim), 0))


def map_key_and_layout(torch_key: str, array: np.ndarray):
    """Upstream key -> ``(converted_key, converted_array)`` or ``None`` if not a network parameter."""
    parts = torch_key.split(".")
    if "all_modules" in parts:
        return None
    n = len(parts)

    def conv_or_plain(module: str, parameter: str) -> np.ndarray:
        return _conv_layout(array) if module == "conv" and parameter == "weight" else array

    if parts[:2] == ["encoder", "stages"] and n == 8 and parts[3].isdigit() and parts[4] == "convs":
        key = f"enc{int(parts[2])}.block{int(parts[5])}.{parts[6]}.{parts[7]}"
        return key, conv_or_plain(parts[6], parts[7])
    if torch_key.startswith("encoder.stem.convs.0.") and n == 6:
        return f"stem.{parts[4]}.{parts[5]}", conv_or_plain(parts[4], parts[5])
    if parts[:2] == ["encoder", "stages"] and n == 8 and parts[3] == "blocks" and parts[5] in ("conv1", "conv2", "conv3"):
        key = f"res{int(parts[2])}.block{int(parts[4])}.{parts[5]}.{parts[6]}.{parts[7]}"
        return key, conv_or_plain(parts[6], parts[7])
    if parts[:2] == ["encoder", "stages"] and n == 9 and parts[3] == "blocks" and parts[5] == "skip" and parts[6].isdigit():
        key = f"res{int(parts[2])}.block{int(parts[4])}.proj.{parts[7]}.{parts[8]}"
        return key, conv_or_plain(parts[7], parts[8])
    if parts[:2] == ["decoder", "stages"] and n == 7:
        key = f"dec{int(parts[2])}.block{int(parts[4])}.{parts[5]}.{parts[6]}"
        return key, conv_or_plain(parts[5], parts[6])
    if parts[:2] == ["decoder", "transpconvs"] and n == 4:
        stage, parameter = int(parts[2]), parts[3]
        return f"up{stage}.{parameter}", (_transposed_layout(array) if parameter == "weight" else array)
    if parts[:2] == ["decoder", "seg_layers"] and n == 4:
        stage, parameter = int(parts[2]), parts[3]
        return f"seg{stage}.{parameter}", (_conv_layout(array) if parameter == "weight" else array)
    return None


def convert_state_dict(state: Mapping[str, object]) -> ConvertedState:
    """Convert an upstream ``state_dict`` (tensors or arrays) to the converted layout."""
    converted: dict[str, np.ndarray] = {}
    dropped: list[str] = []
    for key, value in state.items():
        array = np.asarray(value.detach().cpu().numpy() if hasattr(value, "detach") else value,
                           dtype=np.float32)
        if not np.isfinite(array).all():
            raise ContractError(f"nnU-Net parameter {key!r} contains non-finite values")
        mapped = map_key_and_layout(key, array)
        if mapped is None:
            if key.startswith("decoder.encoder.") or "all_modules" in key:
                dropped.append(key)
                continue
            raise ContractError(f"unsupported nnU-Net checkpoint key {key!r}")
        name, out = mapped
        if name in converted:
            raise ContractError(f"duplicate converted key {name!r}")
        converted[name] = np.ascontiguousarray(out, dtype=np.float32)
    if not converted:
        raise ContractError("checkpoint did not contain convertible weights")
    return ConvertedState(converted, tuple(sorted(dropped)))


def _conv_norm_shapes(shapes: dict, prefix: str, cin: int, cout: int, kernel, spec, *, bias: bool) -> None:
    shapes[f"{prefix}.conv.weight"] = (cout, *kernel, cin)
    if bias:
        shapes[f"{prefix}.conv.bias"] = (cout,)
    if spec.norm_affine:
        shapes[f"{prefix}.norm.weight"] = (cout,)
        shapes[f"{prefix}.norm.bias"] = (cout,)


def expected_shapes(spec: NetworkSpec) -> dict[str, tuple[int, ...]]:
    """Every converted parameter name and shape of a network built from ``spec``, in build order."""
    shapes: dict[str, tuple[int, ...]] = {}
    unit = (1,) * spec.spatial_dims
    if isinstance(spec, ResidualEncoderUNetSpec):
        stem = spec.effective_stem_channels
        _conv_norm_shapes(shapes, "stem", spec.input_channels, stem, spec.kernel_sizes[0], spec,
                          bias=spec.conv_bias)
        cin = stem
        for s, f in enumerate(spec.features):
            k = spec.kernel_sizes[s]
            for b in range(spec.encoder_blocks[s]):
                bin_ = cin if b == 0 else f
                stride = spec.strides[s] if b == 0 else unit
                p = f"res{s}.block{b}"
                if spec.bottleneck_channels is None:
                    _conv_norm_shapes(shapes, f"{p}.conv1", bin_, f, k, spec, bias=spec.conv_bias)
                    _conv_norm_shapes(shapes, f"{p}.conv2", f, f, k, spec, bias=spec.conv_bias)
                else:
                    mid = spec.bottleneck_channels[s]
                    _conv_norm_shapes(shapes, f"{p}.conv1", bin_, mid, unit, spec, bias=spec.conv_bias)
                    _conv_norm_shapes(shapes, f"{p}.conv2", mid, mid, k, spec, bias=spec.conv_bias)
                    _conv_norm_shapes(shapes, f"{p}.conv3", mid, f, unit, spec, bias=spec.conv_bias)
                if bin_ != f:
                    _conv_norm_shapes(shapes, f"{p}.proj", bin_, f, unit, spec, bias=False)
                del stride
            cin = f
    else:
        cin = spec.input_channels
        for s, f in enumerate(spec.features):
            for b in range(spec.encoder_convs[s]):
                _conv_norm_shapes(shapes, f"enc{s}.block{b}", cin if b == 0 else f, f,
                                  spec.kernel_sizes[s], spec, bias=spec.conv_bias)
            cin = f
    stages = len(spec.features)
    for d in range(stages - 1):
        src = stages - 1 - d
        below, skip = spec.features[src], spec.features[src - 1]
        shapes[f"up{d}.weight"] = (skip, *spec.strides[src], below)
        if spec.conv_bias:
            shapes[f"up{d}.bias"] = (skip,)
        for b in range(spec.decoder_convs[d]):
            _conv_norm_shapes(shapes, f"dec{d}.block{b}", 2 * skip if b == 0 else skip, skip,
                              spec.kernel_sizes[src - 1], spec, bias=spec.conv_bias)
        shapes[f"seg{d}.weight"] = (spec.num_classes, *unit, skip)
        shapes[f"seg{d}.bias"] = (spec.num_classes,)
    return shapes


def validate_weights(spec: NetworkSpec, weights: Mapping[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Strict load check: exact key set, shapes, float32 and finite."""
    shapes = expected_shapes(spec)
    missing = sorted(set(shapes) - set(weights))
    extra = sorted(set(weights) - set(shapes))
    if missing or extra:
        raise ContractError(f"checkpoint keys do not match the network: missing {missing[:5]}, "
                            f"unexpected {extra[:5]}")
    out = {}
    for key, shape in shapes.items():
        array = np.ascontiguousarray(weights[key], dtype=np.float32)
        if tuple(array.shape) != shape:
            raise ContractError(f"parameter {key!r} has shape {array.shape}, expected {shape}")
        if not np.isfinite(array).all():
            raise ContractError(f"parameter {key!r} contains non-finite values")
        out[key] = array
    return out
