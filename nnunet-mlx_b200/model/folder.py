"""Load a converted model folder into resident B200 networks (one per fold).

Mirrors reference ``src/nnunet_mlx/model/folder.py``: ``ModelBundle`` (38-62),
``load_model_bundle`` (87-227) and ``auto_detect_folds`` (230-240).  The
folder layout is the reference's: ``plans.json``, ``dataset.json`` and
``fold_<n>/<checkpoint_name>/{state.json, weights.safetensors}``.

Difference by design: the reference keeps one resident network and swaps fold
weights on demand (``model/residency.py``); here every fold keeps its own
weights resident in HBM (31 M parameters = 125 MB per fold), so a fold
ensemble needs no reloads inside the tile loop.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.network import build_network
from nnunet_mlx_b200.model.topology import PlainConvUNetSpec, ResidualEncoderUNetSpec
from nnunet_mlx_b200.storage.checkpoint import load_inference_checkpoint, weights_signature


@dataclass(frozen=True)
class CheckpointProvenance:
    fold: int | str
    checkpoint: str
    weights_signature: list[int]


@dataclass(frozen=True)
class ModelBundle:
    folder: Path
    plans: dict
    dataset_json: dict
    configuration: str
    patch_size: tuple[int, ...]
    spec: PlainConvUNetSpec | ResidualEncoderUNetSpec
    models: tuple
    folds: tuple
    checkpoints: tuple
    mirroring_axes: tuple[int, ...]
    output_channels: int
    regions_class_order: tuple[int, ...] | None
    image_channels: int


def _read_json(path: Path) -> dict:
    if not path.is_file():
        raise ContractError(f"missing {path.name} in model folder")
    try:
        value = json.loads(path.read_text(encoding="utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as error:
        raise ContractError(f"{path.name} is invalid JSON") from error
    if not isinstance(value, dict):
        raise ContractError(f"{path.name} must contain a JSON object")
    return value


def _label_semantics(dataset_json: dict) -> tuple[int, tuple[int, ...] | None]:
    labels = dataset_json.get("labels")
    if not isinstance(labels, dict) or not labels:
        raise ContractError("dataset.json labels must be a non-empty mapping")
    regions = dataset_json.get("regions_class_order")
    if regions is not None:
        order = tuple(int(v) for v in regions)
        return len(order), order
    values = [v for v in labels.values() if not isinstance(v, (list, tuple))]
    if len(values) != len(labels):
        raise ContractError("region-based labels require regions_class_order")
    return len(labels), None


def auto_detect_folds(model_folder: str | Path, *, checkpoint_name: str) -> tuple[int, ...]:
    folder = Path(model_folder)
    found = sorted(int(p.name[5:]) for p in folder.glob("fold_*")
                   if p.name[5:].isdigit() and (p / checkpoint_name).is_dir())
    if not found:
        raise ContractError(f"no numeric folds contain checkpoint {checkpoint_name!r}")
    return tuple(found)


def _spec_from_plans(plans: dict, configuration: str, input_channels: int, num_classes: int):
    try:
        name = plans["configurations"][configuration]["architecture"]["network_class_name"]
    except (KeyError, TypeError) as error:
        raise ContractError(f"nnU-Net plans lack configuration {configuration!r}") from error
    cls = ResidualEncoderUNetSpec if str(name).endswith(".ResidualEncoderUNet") else PlainConvUNetSpec
    return cls.from_plans(plans, configuration=configuration, input_channels=input_channels,
                          num_classes=num_classes)


def load_model_bundle(model_folder: str | Path, *, configuration: str, folds=None,
                      checkpoint_name: str = "checkpoint_final", precision: str = "fp32",
                      device="cuda") -> ModelBundle:
    """Verify a converted model folder and load every selected fold onto ``device``."""
    folder = Path(model_folder)
    if not folder.is_dir():
        raise ContractError(f"model folder does not exist: {folder}")
    plans = _read_json(folder / "plans.json")
    dataset_json = _read_json(folder / "dataset.json")
    channels = dataset_json.get("channel_names") or dataset_json.get("modality")
    if not isinstance(channels, dict) or not channels:
        raise ContractError("dataset.json channel_names must be a non-empty mapping")
    output_channels, regions = _label_semantics(dataset_json)
    spec = _spec_from_plans(plans, configuration, len(channels), output_channels)
    patch = tuple(int(v) for v in plans["configurations"][configuration]["patch_size"])
    if len(patch) != spec.spatial_dims:
        raise ContractError("plan patch_size rank does not match the network")
    selected = auto_detect_folds(folder, checkpoint_name=checkpoint_name) if folds is None else tuple(
        f if f == "all" else int(f) for f in folds)
    if not selected:
        raise ContractError("no folds selected")
    models, provenance, mirrors = [], [], []
    for fold in selected:
        checkpoint = folder / f"fold_{fold}" / checkpoint_name
        if checkpoint.is_file() or checkpoint.suffix == ".pth":
            raise ContractError("checkpoint must be a converted safetensors directory")
        state, weights = load_inference_checkpoint(checkpoint)
        if state.identity.configuration != configuration or state.identity.fold != fold:
            raise ContractError("checkpoint configuration or fold does not match its folder")
        models.append(build_network(spec, precision=precision, device=device).load_weights(weights))
        provenance.append(CheckpointProvenance(fold, checkpoint_name, weights_signature(checkpoint)))
        mirrors.append(state.inference_allowed_mirroring_axes)
    if any(m != mirrors[0] for m in mirrors[1:]):
        raise ContractError("model folds disagree on inference mirroring axes")
    return ModelBundle(folder=folder, plans=plans, dataset_json=dataset_json, configuration=configuration,
                       patch_size=patch, spec=spec, models=tuple(models), folds=selected,
                       checkpoints=tuple(provenance), mirroring_axes=mirrors[0],
                       output_channels=output_channels, regions_class_order=regions,
                       image_channels=len(channels))
