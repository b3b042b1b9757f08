"""Convert trained upstream nnU-Net v2 model folders into converted (safetensors) model folders.

Drop-in for reference ``src/nnunet_mlx/storage/upstream.py``: ``load_upstream_checkpoint``
(94-145), ``detect_upstream_folds`` (148-166), ``convert_trained_model`` (169-297),
``resolve_results_folder`` (300-325) and ``cached_conversion`` (328-367).

An upstream trained model folder is what ``nnUNetv2_train`` leaves under
``nnUNet_results/<dataset>/<trainer>__<plans>__<configuration>``: ``plans.json``,
``dataset.json`` and ``fold_<n>/checkpoint_final.pth``.  Each checkpoint is read
with torch's restricted unpickler (``weights_only=True``, plus NumPy scalar and
dtype reconstructors, which nnU-Net's training log stores); its
``network_weights`` are renamed and re-laid-out to the converted layout
(``storage.weights.convert_state_dict``), checked against the network the plans
describe, and written as ``fold_<n>/checkpoint_final/{weights.safetensors,
state.json}`` beside copies of the two JSON files and a conversion manifest.
Conversion runs on the host and needs no GPU.
"""

from __future__ import annotations

import json
import os
import pickle
import re
import shutil
import tempfile
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.storage.checkpoint import (
    CheckpointIdentity,
    InferenceCheckpointState,
    read_state,
    read_weights,
    save_inference_checkpoint,
)
from nnunet_mlx_b200.storage.weights import convert_state_dict, validate_weights

UPSTREAM_CHECKPOINT = "checkpoint_final.pth"
CONVERTED_CHECKPOINT = "checkpoint_final"
CONVERSION_FILENAME = "conversion.json"
CONVERSION_SCHEMA = "nnunet-mlx.conversion.v1"
CONVERSION_CONTRACT_VERSION = 1
RESULTS_VARIABLE = "nnUNet_results"   # nnU-Net's own environment variable name
CACHE_VARIABLE = "NNUNET_MLX_CACHE"

# Trainers whose inference network is the one plans.json describes (they change only
# optimisation, loss, augmentation, epochs or mirroring); the names are upstream's.
PLANS_BUILT_TRAINERS = (
    "nnUNetTrainer",
    "nnUNetTrainerAdam", "nnUNetTrainerAdam1en3", "nnUNetTrainerAdam3en4",
    "nnUNetTrainerAdan", "nnUNetTrainerAdan1en1", "nnUNetTrainerAdan1en3",
    "nnUNetTrainerAdan3en4", "nnUNetTrainerAdanCosAnneal",
    "nnUNetTrainerBenchmark_5epochs", "nnUNetTrainerBenchmark_5epochs_noDataLoading",
    "nnUNetTrainerCELoss", "nnUNetTrainerCELoss_5epochs", "nnUNetTrainerCosAnneal",
    "nnUNetTrainerDA5", "nnUNetTrainerDA5Segord0", "nnUNetTrainerDA5_10epochs",
    "nnUNetTrainerDA5ord0", "nnUNetTrainerDiceCELoss_noSmooth", "nnUNetTrainerDiceLoss",
    "nnUNetTrainerDiceTopK10Loss", "nnUNetTrainerNoDA", "nnUNetTrainerNoDeepSupervision",
    "nnUNetTrainerNoMirroring", "nnUNetTrainerTopk10Loss", "nnUNetTrainerTopk10LossLS01",
    "nnUNetTrainerVanillaAdam", "nnUNetTrainerVanillaAdam1en3", "nnUNetTrainerVanillaAdam3en4",
    "nnUNetTrainer_1epoch", "nnUNetTrainer_5epochs", "nnUNetTrainer_10epochs",
    "nnUNetTrainer_20epochs", "nnUNetTrainer_50epochs", "nnUNetTrainer_100epochs",
    "nnUNetTrainer_250epochs", "nnUNetTrainer_500epochs", "nnUNetTrainer_750epochs",
    "nnUNetTrainer_2000epochs", "nnUNetTrainer_4000epochs", "nnUNetTrainer_8000epochs",
    "nnUNetTrainer_250epochs_NoMirroring", "nnUNetTrainer_2000epochs_NoMirroring",
    "nnUNetTrainer_4000epochs_NoMirroring", "nnUNetTrainer_8000epochs_NoMirroring",
    "nnUNetTrainer_DASegOrd0", "nnUNetTrainer_DASegOrd0_NoMirroring",
)


@dataclass(frozen=True, slots=True)
class UpstreamCheckpoint:
    """What inference needs from an upstream ``checkpoint_final.pth``; ``mirroring_axes``
    is the trainer's ``inference_allowed_mirroring_axes`` (``None`` -> ``()``)."""

    network_weights: dict[str, object]
    trainer_name: str
    configuration: str
    mirroring_axes: tuple[int, ...]
    current_epoch: int | None


@dataclass(frozen=True, slots=True)
class ConversionResult:
    folder: Path
    configuration: str
    trainer_name: str
    folds: tuple[int | str, ...]


def _safe_globals() -> list[object]:
    """NumPy reconstructors nnU-Net checkpoints need beyond tensors and containers."""
    try:
        from numpy._core.multiarray import scalar
    except ImportError:  # NumPy < 2
        from numpy.core.multiarray import scalar
    dtypes = (np.bool_, np.int8, np.int16, np.int32, np.int64, np.uint8, np.uint16, np.uint32, np.uint64,
              np.float16, np.float32, np.float64, np.complex64, np.complex128)
    return [scalar, (scalar, "numpy.core.multiarray.scalar"), np.dtype, *(type(np.dtype(t)) for t in dtypes)]


def _int(value, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, (int, np.integer)):
        raise ContractError(f"{name} must be an integer")
    return int(value)


def load_upstream_checkpoint(path: str | Path) -> UpstreamCheckpoint:
    """Read an upstream nnU-Net checkpoint with torch's restricted unpickler."""
    import torch
    import torch.serialization

    source = Path(path)
    if not source.is_file():
        raise ContractError(f"upstream checkpoint does not exist: {source}")
    with torch.serialization.safe_globals(_safe_globals()):
        try:
            raw = torch.load(source, map_location="cpu", weights_only=True)
        except (pickle.UnpicklingError, RuntimeError, EOFError, OSError) as error:
            raise ContractError(f"cannot read upstream checkpoint {source}: {error}") from error
    if not isinstance(raw, dict):
        raise ContractError(f"{source.name} is not a checkpoint mapping")
    weights = raw.get("network_weights")
    init_args = raw.get("init_args")
    trainer = raw.get("trainer_name")
    if not isinstance(weights, dict) or not weights:
        raise ContractError(f"{source.name} has no network_weights")
    if not isinstance(init_args, dict) or not isinstance(init_args.get("configuration"), str):
        raise ContractError(f"{source.name} has no init_args.configuration")
    if not isinstance(trainer, str) or not trainer:
        raise ContractError(f"{source.name} has no trainer_name")
    axes = raw.get("inference_allowed_mirroring_axes")
    if axes is not None and not isinstance(axes, (list, tuple)):
        raise ContractError("inference_allowed_mirroring_axes must be a sequence or None")
    epoch = raw.get("current_epoch")
    return UpstreamCheckpoint(
        network_weights=dict(weights), trainer_name=trainer, configuration=init_args["configuration"],
        mirroring_axes=() if axes is None else tuple(_int(a, "mirroring axis") for a in axes),
        current_epoch=None if epoch is None else _int(epoch, "current_epoch"))


def detect_upstream_folds(model_folder: str | Path, *,
                          checkpoint_name: str = UPSTREAM_CHECKPOINT) -> tuple[int | str, ...]:
    """Numeric folds (sorted), then ``"all"``, whose ``fold_*`` folder holds ``checkpoint_name``."""
    folder = Path(model_folder)
    numeric, has_all = [], False
    for candidate in folder.glob("fold_*"):
        if not (candidate / checkpoint_name).is_file():
            continue
        suffix = candidate.name.removeprefix("fold_")
        if suffix.isdigit() and str(int(suffix)) == suffix:
            numeric.append(int(suffix))
        elif suffix == "all":
            has_all = True
    folds: tuple[int | str, ...] = (*sorted(numeric), *(("all",) if has_all else ()))
    if not folds:
        raise ContractError(f"no fold_* folder in {folder} contains {checkpoint_name}")
    return folds


def _validate_folds(folds) -> tuple[int | str, ...]:
    out: list[int | str] = []
    for fold in folds:
        if fold == "all":
            out.append("all")
        elif isinstance(fold, str) and fold.isdigit():
            out.append(int(fold))
        elif isinstance(fold, int) and not isinstance(fold, bool) and fold >= 0:
            out.append(fold)
        else:
            raise ContractError(f"invalid fold {fold!r}")
    if not out or len(set(out)) != len(out):
        raise ContractError("folds must be a non-empty list without duplicates")
    return tuple(out)


def _read_json(path: Path) -> dict:
    try:
        value = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as error:
        raise ContractError(f"cannot read {path}: {error}") from error
    if not isinstance(value, dict):
        raise ContractError(f"{path} must hold a JSON object")
    return value


def _planned_spec(plans: dict, dataset_json: dict, configuration: str):
    from nnunet_mlx_b200.model.folder import _label_semantics, _spec_from_plans

    channels = dataset_json.get("channel_names") or dataset_json.get("modality")
    if not isinstance(channels, dict) or not channels:
        raise ContractError("dataset.json channel_names must be a non-empty mapping")
    output_channels, _ = _label_semantics(dataset_json)
    if configuration not in plans.get("configurations", {}):
        raise ContractError(f"plans.json has no configuration {configuration!r}")
    return _spec_from_plans(plans, configuration, len(channels), output_channels)


def convert_trained_model(source: str | Path, destination: str | Path, *, folds: Sequence[int | str] | None = None,
                          checkpoint_name: str = UPSTREAM_CHECKPOINT) -> ConversionResult:
    """Convert a trained upstream model folder into a new converted model folder.

    Every fold must come from the same plans-built trainer and configuration and
    its weights must map exactly onto the network ``plans.json`` describes.  The
    folder is written to a staging directory, read back, and only then moved to
    ``destination`` (which must not exist).
    """
    folder = Path(source)
    if not folder.is_dir():
        raise ContractError(f"trained model folder does not exist: {folder}")
    if Path(checkpoint_name).name != checkpoint_name:
        raise ContractError("checkpoint name must be a file name")
    target = Path(destination)
    if target.exists():
        raise ContractError(f"conversion destination exists: {target}")
    plans = _read_json(folder / "plans.json")
    dataset_json = _read_json(folder / "dataset.json")
    selected = detect_upstream_folds(folder, checkpoint_name=checkpoint_name) if folds is None \
        else _validate_folds(folds)
    paths = [folder / f"fold_{fold}" / checkpoint_name for fold in selected]
    first = load_upstream_checkpoint(paths[0])
    if first.trainer_name not in PLANS_BUILT_TRAINERS:
        raise ContractError(f"trainer {first.trainer_name!r} is not supported: only trainers that build the "
                            "network from plans.json can be converted")
    configuration = first.configuration
    spec = _planned_spec(plans, dataset_json, configuration)
    target.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{target.name}.", dir=target.parent))
    try:
        shutil.copyfile(folder / "plans.json", staging / "plans.json")
        shutil.copyfile(folder / "dataset.json", staging / "dataset.json")
        entries = []
        for fold, path in zip(selected, paths):
            checkpoint = first if path == paths[0] else load_upstream_checkpoint(path)
            if (checkpoint.trainer_name, checkpoint.configuration) != (first.trainer_name, configuration):
                raise ContractError(f"fold {fold} was trained with a different trainer or configuration "
                                    "than the other folds")
            converted = convert_state_dict(checkpoint.network_weights)
            try:
                weights = validate_weights(spec, converted.weights)
            except ContractError as error:
                raise ContractError(f"fold {fold} weights do not match the network planned in plans.json: "
                                    f"{error}") from error
            state = InferenceCheckpointState(
                identity=CheckpointIdentity(checkpoint.trainer_name, configuration, fold),
                current_epoch=checkpoint.current_epoch, spatial_dims=spec.spatial_dims,
                inference_allowed_mirroring_axes=checkpoint.mirroring_axes,
                dropped_source_keys=converted.dropped_keys)
            save_inference_checkpoint(staging / f"fold_{fold}" / CONVERTED_CHECKPOINT, weights=weights, state=state)
            stat = path.stat()
            entries.append({"fold": fold, "checkpoint": CONVERTED_CHECKPOINT, "source_checkpoint": checkpoint_name,
                            "source_size_bytes": stat.st_size, "source_mtime_ns": stat.st_mtime_ns})
        manifest = {"schema_version": CONVERSION_SCHEMA, "conversion_contract_version": CONVERSION_CONTRACT_VERSION,
                    "source_plans": plans, "source_dataset": dataset_json, "configuration": configuration,
                    "trainer_name": first.trainer_name, "architecture": type(spec).__name__,
                    "spatial_dims": spec.spatial_dims, "folds": entries}
        (staging / CONVERSION_FILENAME).write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n",
                                                   encoding="utf-8")
        # read back what was written
        for fold in selected:
            directory = staging / f"fold_{fold}" / CONVERTED_CHECKPOINT
            state = read_state(directory)
            if state.identity.fold != fold or state.identity.configuration != configuration:
                raise ContractError(f"converted fold {fold} does not read back")
            validate_weights(spec, read_weights(directory))
        staging.rename(target)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise
    return ConversionResult(target, configuration, first.trainer_name, selected)


def read_conversion_manifest(folder: str | Path) -> dict:
    manifest = _read_json(Path(folder) / CONVERSION_FILENAME)
    if manifest.get("schema_version") != CONVERSION_SCHEMA:
        raise ContractError(f"{folder} is not a conversion of this schema")
    if not isinstance(manifest.get("configuration"), str) or not isinstance(manifest.get("folds"), list):
        raise ContractError(f"{folder}: malformed conversion manifest")
    return manifest


def resolve_results_folder(dataset: str, *, configuration: str, trainer: str = "nnUNetTrainer",
                           plans: str = "nnUNetPlans", results: str | Path | None = None) -> Path:
    """``<results>/<dataset>/<trainer>__<plans>__<configuration>`` as nnU-Net lays it out; ``dataset``
    is an ID (``3`` -> the one ``Dataset003_*`` folder) or a full name; ``results`` defaults to
    ``$nnUNet_results``."""
    root_value = results if results is not None else os.environ.get(RESULTS_VARIABLE)
    if not root_value:
        raise ContractError(f"set {RESULTS_VARIABLE}, or pass a trained model folder with -m")
    root = Path(root_value).expanduser()
    if dataset.isdigit():
        pattern = re.compile(rf"Dataset{int(dataset):03d}_.+")
        matches = sorted(p.name for p in root.glob("Dataset*") if p.is_dir() and pattern.fullmatch(p.name))
        if len(matches) != 1:
            raise ContractError(f"expected one Dataset{int(dataset):03d}_* folder in {root}, found {len(matches)}")
        dataset = matches[0]
    folder = root / dataset / f"{trainer}__{plans}__{configuration}"
    if not folder.is_dir():
        raise ContractError(f"trained model folder does not exist: {folder}")
    return folder


def _conversion_is_current(target: Path, folder: Path, folds: tuple[int | str, ...], checkpoint_name: str) -> bool:
    marker = target / ".source"
    if not marker.is_file() or marker.read_text(encoding="utf-8").strip() != str(folder):
        return False
    try:
        manifest = read_conversion_manifest(target)
        if (manifest.get("conversion_contract_version") != CONVERSION_CONTRACT_VERSION
                or manifest.get("source_plans") != _read_json(folder / "plans.json")
                or manifest.get("source_dataset") != _read_json(folder / "dataset.json")):
            return False
    except ContractError:
        return False
    recorded = {entry.get("fold"): (entry.get("source_checkpoint"), entry.get("source_size_bytes"),
                                    entry.get("source_mtime_ns"))
                for entry in manifest["folds"] if isinstance(entry, dict)}
    if set(recorded) != set(folds):
        return False
    for fold in folds:
        stat = (folder / f"fold_{fold}" / checkpoint_name).stat()
        if recorded[fold] != (checkpoint_name, stat.st_size, stat.st_mtime_ns):
            return False
        if not (target / f"fold_{fold}" / CONVERTED_CHECKPOINT / "weights.safetensors").is_file():
            return False
    return True


def cached_conversion(trained_folder: str | Path, *, folds: Sequence[int | str] | None = None,
                      checkpoint_name: str = UPSTREAM_CHECKPOINT, cache: str | Path | None = None) -> Path:
    """A converted copy of ``trained_folder`` under ``$NNUNET_MLX_CACHE`` (default
    ``~/.cache/nnunet-mlx``)/``converted/<dataset>/<model>``, rebuilt when the source plans, dataset or
    any fold checkpoint (size, mtime) changed.  Every available fold is converted."""
    folder = Path(trained_folder).absolute()
    available = detect_upstream_folds(folder, checkpoint_name=checkpoint_name)
    wanted = available if folds is None else _validate_folds(folds)
    missing = [fold for fold in wanted if fold not in available]
    if missing:
        raise ContractError(f"folds {missing} have no {checkpoint_name} in {folder}")
    root = Path(cache or os.environ.get(CACHE_VARIABLE, "~/.cache/nnunet-mlx")).expanduser()
    normalized = Path(os.path.normpath(str(folder)))
    if not normalized.name or not normalized.parent.name:
        raise ContractError("trained folder needs dataset and model directory names")
    target = root / "converted" / normalized.parent.name / normalized.name
    if target.is_symlink():
        raise ContractError(f"conversion cache entry must not be a symlink: {target}")
    if _conversion_is_current(target, folder, available, checkpoint_name):
        return target
    if target.exists():
        shutil.rmtree(target)
    convert_trained_model(folder, target, folds=available, checkpoint_name=checkpoint_name)
    (target / ".source").write_text(str(folder) + "\n", encoding="utf-8")
    return target
