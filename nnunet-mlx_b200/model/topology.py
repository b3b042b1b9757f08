"""Network topology specs parsed from nnU-Net plans.

Same field names, defaults and validation outcomes as reference
``src/nnunet_mlx/model/topology.py`` (``PlainConvUNetSpec`` 132-254,
``ResidualEncoderUNetSpec`` 257-430), so plans that the reference admits build
the same networks here, and plans it rejects raise ``ContractError`` here too.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass

from nnunet_mlx_b200.errors import ContractError

SpatialShape = tuple[int, ...]


def _mapping(value: object, name: str) -> Mapping[str, object]:
    if not isinstance(value, Mapping):
        raise ContractError(f"{name} must be a mapping")
    return value


def _sequence(value: object, name: str) -> Sequence[object]:
    if isinstance(value, (str, bytes)) or not isinstance(value, Sequence):
        raise ContractError(f"{name} must be a sequence")
    return value


def _positive_int(value: object, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < 1:
        raise ContractError(f"{name} must be a positive integer")
    return value


def _positive_ints(value: object, name: str) -> tuple[int, ...]:
    result = tuple(_positive_int(v, name) for v in _sequence(value, name))
    if not result:
        raise ContractError(f"{name} must not be empty")
    return result


def _boolean(value: object, name: str) -> bool:
    if not isinstance(value, bool):
        raise ContractError(f"{name} must be a boolean")
    return value


def _number(value: object, name: str) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise ContractError(f"{name} must be a number")
    return float(value)


def _spatial_rows(value: object, name: str) -> tuple[SpatialShape, ...]:
    rows = tuple(_positive_ints(row, name) for row in _sequence(value, name))
    dims = {len(r) for r in rows}
    if not rows or len(dims) != 1 or next(iter(dims)) not in (2, 3):
        raise ContractError(f"{name} rows must use one 2-D or 3-D dimensionality")
    return rows


def _validate_ops(kwargs: Mapping[str, object], spatial_dims: int) -> None:
    conv, norm, nonlin = kwargs.get("conv_op"), kwargs.get("norm_op"), kwargs.get("nonlin")
    if not isinstance(conv, str) or not conv.endswith(f".Conv{spatial_dims}d"):
        raise ContractError(f"{spatial_dims}-D nnU-Net requires Conv{spatial_dims}d, got {conv!r}")
    if not isinstance(norm, str) or not norm.endswith(f".InstanceNorm{spatial_dims}d"):
        raise ContractError(f"{spatial_dims}-D nnU-Net requires InstanceNorm{spatial_dims}d, got {norm!r}")
    if not isinstance(nonlin, str) or not nonlin.endswith(".LeakyReLU"):
        raise ContractError(f"{spatial_dims}-D nnU-Net requires LeakyReLU, got {nonlin!r}")


def _validate_semantics(kwargs: Mapping[str, object]) -> None:
    if _boolean(kwargs.get("nonlin_first", False), "nonlin_first"):
        raise ContractError("unsupported nonlin_first activation ordering")
    stages = len(_sequence(kwargs.get("features_per_stage"), "features_per_stage"))
    if "n_stages" in kwargs and _positive_int(kwargs["n_stages"], "n_stages") != stages:
        raise ContractError("n_stages does not match features_per_stage")
    dropout = kwargs.get("dropout_op")
    if dropout is not None:
        if not isinstance(dropout, str) or dropout.rsplit(".", 1)[-1] not in {"Dropout", "Dropout2d", "Dropout3d"}:
            raise ContractError("unsupported dropout_op")
        options = _mapping(kwargs.get("dropout_op_kwargs"), "dropout_op_kwargs")
        if _number(options.get("p", 0.5), "dropout p") != 0:
            raise ContractError("unsupported nonzero dropout")
        if set(options) - {"p", "inplace"}:
            raise ContractError("unsupported dropout options")
    norm = _mapping(kwargs.get("norm_op_kwargs", {}), "norm_op_kwargs")
    if set(norm) - {"eps", "affine", "momentum", "track_running_stats"}:
        raise ContractError("unsupported normalization options")
    if _boolean(norm.get("track_running_stats", False), "track_running_stats"):
        raise ContractError("unsupported normalization running statistics")
    nonlin = _mapping(kwargs.get("nonlin_kwargs", {}), "nonlin_kwargs")
    if set(nonlin) - {"negative_slope", "inplace"}:
        raise ContractError("unsupported activation options")


def _architecture(plans: Mapping[str, object], configuration: str, suffix: str) -> Mapping[str, object]:
    configurations = _mapping(plans.get("configurations"), "configurations")
    raw = configurations.get(configuration)
    if raw is None:
        raise ContractError(f"nnU-Net plans lack configuration {configuration!r}")
    architecture = _mapping(_mapping(raw, configuration).get("architecture"), "architecture")
    name = architecture.get("network_class_name")
    if not isinstance(name, str) or not name.endswith(suffix):
        raise ContractError(f"unsupported nnU-Net architecture {name!r}")
    kwargs = _mapping(architecture.get("arch_kwargs"), "arch_kwargs")
    _validate_semantics(kwargs)
    return kwargs


def _common_checks(spec, stages_field: tuple[int, ...], kind: str) -> None:
    stages = len(spec.features)
    if spec.input_channels < 1 or spec.num_classes < 1:
        raise ContractError(f"{kind} needs input channels and at least one output")
    if stages < 2:
        raise ContractError(f"{kind} needs at least two stages")
    if any(n != stages for n in (len(spec.kernel_sizes), len(spec.strides), len(stages_field))):
        raise ContractError("encoder topology lengths do not match")
    if len(spec.decoder_convs) != stages - 1:
        raise ContractError("decoder topology must have one entry per skip connection")
    dims = {len(row) for row in (*spec.kernel_sizes, *spec.strides)}
    if len(dims) != 1 or next(iter(dims)) not in (2, 3):
        raise ContractError(f"{kind} requires consistent 2-D or 3-D spatial rows")
    if any(v < 1 or v % 2 == 0 for row in spec.kernel_sizes for v in row):
        raise ContractError("only positive odd convolution kernels are supported")
    if spec.norm_eps <= 0:
        raise ContractError("normalization epsilon must be positive")
    if not 0 <= spec.leaky_slope <= 1:
        raise ContractError("LeakyReLU negative_slope must be in [0, 1]")


@dataclass(frozen=True, slots=True)
class PlainConvUNetSpec:
    """Upstream ``PlainConvUNet`` topology (reference topology.py:132-254)."""

    input_channels: int
    num_classes: int
    features: tuple[int, ...]
    kernel_sizes: tuple[SpatialShape, ...]
    strides: tuple[SpatialShape, ...]
    encoder_convs: tuple[int, ...]
    decoder_convs: tuple[int, ...]
    conv_bias: bool = True
    norm_eps: float = 1e-5
    norm_affine: bool = True
    leaky_slope: float = 0.01

    def __post_init__(self) -> None:
        _common_checks(self, self.encoder_convs, "PlainConvUNet")

    @property
    def spatial_dims(self) -> int:
        return len(self.kernel_sizes[0])

    @classmethod
    def from_plans(cls, plans, *, configuration: str, input_channels: int, num_classes: int):
        kwargs = _architecture(plans, configuration, ".PlainConvUNet")
        kernel_sizes = _spatial_rows(kwargs.get("kernel_sizes"), "kernel_sizes")
        _validate_ops(kwargs, len(kernel_sizes[0]))
        norm = _mapping(kwargs.get("norm_op_kwargs", {}), "norm_op_kwargs")
        nonlin = _mapping(kwargs.get("nonlin_kwargs", {}), "nonlin_kwargs")
        return cls(
            input_channels=input_channels, num_classes=num_classes,
            features=_positive_ints(kwargs.get("features_per_stage"), "features"),
            kernel_sizes=kernel_sizes,
            strides=_spatial_rows(kwargs.get("strides"), "strides"),
            encoder_convs=_positive_ints(kwargs.get("n_conv_per_stage"), "encoder"),
            decoder_convs=_positive_ints(kwargs.get("n_conv_per_stage_decoder"), "decoder"),
            conv_bias=_boolean(kwargs.get("conv_bias", False), "conv_bias"),
            norm_eps=_number(norm.get("eps", 1e-5), "norm eps"),
            norm_affine=_boolean(norm.get("affine", False), "norm affine"),
            leaky_slope=_number(nonlin.get("negative_slope", 0.01), "leaky slope"),
        )


@dataclass(frozen=True, slots=True)
class ResidualEncoderUNetSpec:
    """Upstream ``ResidualEncoderUNet`` topology (reference topology.py:257-430)."""

    input_channels: int
    num_classes: int
    features: tuple[int, ...]
    kernel_sizes: tuple[SpatialShape, ...]
    strides: tuple[SpatialShape, ...]
    encoder_blocks: tuple[int, ...]
    decoder_convs: tuple[int, ...]
    conv_bias: bool = True
    norm_eps: float = 1e-5
    norm_affine: bool = True
    leaky_slope: float = 0.01
    stem_channels: int | None = None
    bottleneck_channels: tuple[int, ...] | None = None

    def __post_init__(self) -> None:
        _common_checks(self, self.encoder_blocks, "ResidualEncoderUNet")
        if self.stem_channels is not None and self.stem_channels < 1:
            raise ContractError("stem channels must be positive")
        if self.bottleneck_channels is not None:
            if len(self.bottleneck_channels) != len(self.features):
                raise ContractError("bottleneck channels must have one entry per encoder stage")
            if any(c < 1 for c in self.bottleneck_channels):
                raise ContractError("bottleneck channels must be positive")

    @property
    def spatial_dims(self) -> int:
        return len(self.kernel_sizes[0])

    @property
    def effective_stem_channels(self) -> int:
        return self.stem_channels or self.features[0]

    @classmethod
    def from_plans(cls, plans, *, configuration: str, input_channels: int, num_classes: int):
        kwargs = _architecture(plans, configuration, ".ResidualEncoderUNet")
        kernel_sizes = _spatial_rows(kwargs.get("kernel_sizes"), "kernel_sizes")
        _validate_ops(kwargs, len(kernel_sizes[0]))
        features = _positive_ints(kwargs.get("features_per_stage"), "features")
        block = kwargs.get("block")
        raw_bottleneck = kwargs.get("bottleneck_channels")
        if block is None or (isinstance(block, str) and block.endswith(".BasicBlockD")):
            if raw_bottleneck is not None:
                raise ContractError("BasicBlockD plans must not define bottleneck channels")
            bottleneck = None
        elif isinstance(block, str) and block.endswith(".BottleneckD"):
            if raw_bottleneck is None:
                raise ContractError("BottleneckD requires bottleneck channels")
            if isinstance(raw_bottleneck, int) and not isinstance(raw_bottleneck, bool):
                bottleneck = (_positive_int(raw_bottleneck, "bottleneck channels"),) * len(features)
            else:
                bottleneck = _positive_ints(raw_bottleneck, "bottleneck channels")
        else:
            raise ContractError(f"unsupported residual block {block!r}")
        norm = _mapping(kwargs.get("norm_op_kwargs", {}), "norm_op_kwargs")
        nonlin = _mapping(kwargs.get("nonlin_kwargs", {}), "nonlin_kwargs")
        stem = kwargs.get("stem_channels")
        return cls(
            input_channels=input_channels, num_classes=num_classes, features=features,
            kernel_sizes=kernel_sizes,
            strides=_spatial_rows(kwargs.get("strides"), "strides"),
            encoder_blocks=_positive_ints(kwargs.get("n_blocks_per_stage"), "encoder blocks"),
            decoder_convs=_positive_ints(kwargs.get("n_conv_per_stage_decoder"), "decoder"),
            conv_bias=_boolean(kwargs.get("conv_bias", False), "conv_bias"),
            norm_eps=_number(norm.get("eps", 1e-5), "norm eps"),
            norm_affine=_boolean(norm.get("affine", False), "norm affine"),
            leaky_slope=_number(nonlin.get("negative_slope", 0.01), "leaky slope"),
            stem_channels=None if stem is None else _positive_int(stem, "stem channels"),
            bottleneck_channels=bottleneck,
        )


NetworkSpec = PlainConvUNetSpec | ResidualEncoderUNetSpec
