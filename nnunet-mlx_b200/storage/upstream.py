"""Convert trained upstream nnU-Net v2 model folders into converted (safetensors) model folders.

Same public names and arguments as reference ``src/nnunet_mlx/storage/upstream.py``
(``load_upstream_checkpoint``, ``detect_upstream_folds``, ``convert_trained_model``,
``resolve_results_folder``, ``cached_conversion``), so the ``predict -d/-tr/-p/-c``
path resolves and converts the same folders.  The design here:

* ``TrainedModelFolder`` is the upstream folder ``nnUNetv2_train`` leaves under
  ``nnUNet_results/<dataset>/<trainer>__<plans>__<configuration>``
  (``plans.json``, ``dataset.json``, ``fold_<n>/checkpoint_final.pth``): it
  lists its folds and computes a *source fingerprint* -- the parsed plans and
  dataset JSON plus each fold checkpoint's size and modification time.
* Checkpoints are read inspect-then-allow: the pickle's global references are
  listed first (``torch.serialization.get_unsafe_globals_in_checkpoint``); any
  reference outside a fixed table of NumPy reconstructors (the scalar / dtype
  objects nnU-Net's training log pickles) refuses the file before it is
  unpickled, and the load then runs with exactly the references found.
* A conversion is written into a staging folder, read back, and renamed into
  place; the conversion manifest records the source folder and its
  fingerprint.  The cache keeps one converted folder per trained folder and
  rebuilds it when the fingerprint it recorded no longer matches (the new
  folder is completed beside the old one and swapped in).

Conversion runs on the host and needs no GPU.
"""

from __future__ import annotations

import json
import os
import shutil
import tempfile
from collections.abc import Iterable, Sequence
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
DEFAULT_CACHE = "~/.cache/nnunet-mlx"

# Upstream trainer classes that build their inference network from plans.json unchanged (they differ only
# in optimiser, loss, augmentation, epoch count or mirroring), by upstream's class names.  Trainers outside
# this set may build a different network and are refused.
_EPOCH_VARIANTS = (1, 5, 10, 20, 50, 100, 250, 500, 750, 2000, 4000, 8000)
PLANS_BUILT_TRAINERS = frozenset(
    {"nnUNetTrainer", "nnUNetTrainerNoDeepSupervision", "nnUNetTrainerNoMirroring", "nnUNetTrainerNoDA",
     "nnUNetTrainerDA5", "nnUNetTrainerDA5Segord0", "nnUNetTrainerDA5_10epochs", "nnUNetTrainerDA5ord0",
     "nnUNetTrainer_DASegOrd0", "nnUNetTrainer_DASegOrd0_NoMirroring",
     "nnUNetTrainerCELoss", "nnUNetTrainerCELoss_5epochs", "nnUNetTrainerDiceLoss",
     "nnUNetTrainerDiceCELoss_noSmooth", "nnUNetTrainerDiceTopK10Loss", "nnUNetTrainerTopk10Loss",
     "nnUNetTrainerTopk10LossLS01", "nnUNetTrainerCosAnneal", "nnUNetTrainerAdanCosAnneal",
     "nnUNetTrainerBenchmark_5epochs", "nnUNetTrainerBenchmark_5epochs_noDataLoading"}
    | {f"nnUNetTrainer{opt}{lr}" for opt in ("Adam", "VanillaAdam") for lr in ("", "1en3", "3en4")}
    | {f"nnUNetTrainerAdan{lr}" for lr in ("", "1en1", "1en3", "3en4")}
    | {"nnUNetTrainer_1epoch"} | {f"nnUNetTrainer_{n}epochs" for n in _EPOCH_VARIANTS if n > 1}
    | {f"nnUNetTrainer_{n}epochs_NoMirroring" for n in (250, 2000, 4000, 8000)}
)


# ---------------------------------------------------------------------------- restricted checkpoint reading
def _numpy_reconstructors() -> dict[str, object]:
    """Qualified pickle names -> the NumPy objects a checkpoint may reference (scalars, dtypes)."""
    try:
        from numpy._core.multiarray import scalar
    except ImportError:  # NumPy < 2
        from numpy.core.multiarray import scalar
    table: dict[str, object] = {
        "numpy.core.multiarray.scalar": scalar,   # checkpoints pickled under NumPy 1.x
        "numpy._core.multiarray.scalar": scalar,  # and under NumPy 2.x
        "numpy.dtype": np.dtype,
    }
    for code in "?bhilqBHILQefdgFD":
        dtype_class = type(np.dtype(code))
        table[f"numpy.dtypes.{dtype_class.__name__}"] = dtype_class
    return table


def _checked_globals(source: Path) -> list[tuple[object, str]]:
    """The global references of ``source``'s pickle, resolved against the NumPy table; anything else refuses."""
    import torch.serialization

    try:
        names = torch.serialization.get_unsafe_globals_in_checkpoint(source)
    except Exception as error:  # not a torch zip archive, truncated, unreadable
        raise ContractError(f"upstream checkpoint {source} is unreadable: {error}") from error
    table = _numpy_reconstructors()
    refused = sorted(name for name in names if name not in table)
    if refused:
        raise ContractError(f"upstream checkpoint {source} is unreadable: it references {', '.join(refused)}, "
                            "which the restricted load does not allow")
    allowed = [(table[name], name) for name in names]
    if "numpy.dtype" in names:
        # a pickled dtype is rebuilt as an instance of its dtype class, which the scan does not list
        allowed += [(obj, name) for name, obj in table.items() if name.startswith("numpy.dtypes.")]
    return allowed


@dataclass(frozen=True, slots=True)
class UpstreamCheckpoint:
    """What inference needs from an upstream ``checkpoint_final.pth``; ``mirroring_axes``
    is the trainer's ``inference_allowed_mirroring_axes`` (``None`` -> ``()``)."""

    network_weights: dict[str, object]
    trainer_name: str
    configuration: str
    mirroring_axes: tuple[int, ...]
    current_epoch: int | None


def _integer(value, what: str) -> int:
    if isinstance(value, (int, np.integer)) and not isinstance(value, (bool, np.bool_)):
        return int(value)
    raise ContractError(f"{what} must be an integer, got {value!r}")


def load_upstream_checkpoint(path: str | Path) -> UpstreamCheckpoint:
    """Read an upstream nnU-Net checkpoint without running arbitrary pickled code.

    The pickle may reference tensors, plain containers and NumPy scalars /
    dtypes only; the returned record holds the network weights and the fields
    conversion needs.
    """
    import torch
    import torch.serialization

    source = Path(path)
    if not source.is_file():
        raise ContractError(f"upstream checkpoint does not exist: {source}")
    allowed = _checked_globals(source)
    try:
        with torch.serialization.safe_globals(allowed):
            payload = torch.load(source, map_location="cpu", weights_only=True)
    except Exception as error:
        raise ContractError(f"upstream checkpoint {source} is unreadable: {error}") from error
    if not isinstance(payload, dict):
        raise ContractError(f"{source.name}: expected a checkpoint dictionary, got {type(payload).__name__}")

    def field(name, kind, description):
        value = payload.get(name)
        if not isinstance(value, kind) or not value:
            raise ContractError(f"{source.name}: missing or empty {description}")
        return value

    weights = field("network_weights", dict, "network_weights")
    init_args = field("init_args", dict, "init_args")
    trainer = field("trainer_name", str, "trainer_name")
    configuration = init_args.get("configuration")
    if not isinstance(configuration, str) or not configuration:
        raise ContractError(f"{source.name}: init_args carry no configuration name")
    axes = payload.get("inference_allowed_mirroring_axes")
    if axes is not None and not isinstance(axes, (list, tuple)):
        raise ContractError(f"{source.name}: inference_allowed_mirroring_axes must be a sequence or None")
    epoch = payload.get("current_epoch")
    return UpstreamCheckpoint(
        network_weights=dict(weights), trainer_name=trainer, configuration=configuration,
        mirroring_axes=tuple(_integer(a, "a mirroring axis") for a in (axes or ())),
        current_epoch=None if epoch is None else _integer(epoch, "current_epoch"))


# ---------------------------------------------------------------------------- the trained folder
def _fold_from_directory(name: str) -> int | str | None:
    """``fold_3`` -> 3, ``fold_all`` -> "all"; anything else (``fold_03``, ``fold_x``) -> None."""
    if not name.startswith("fold_"):
        return None
    tail = name[len("fold_"):]
    if tail == "all":
        return "all"
    if tail.isdigit() and tail == str(int(tail)):
        return int(tail)
    return None


def _fold_order(fold: int | str) -> tuple[int, int]:
    return (1, 0) if fold == "all" else (0, int(fold))


def _load_json_object(path: Path) -> dict:
    try:
        with path.open(encoding="utf-8") as handle:
            value = json.load(handle)
    except (OSError, ValueError) as error:
        raise ContractError(f"{path} is unreadable: {error}") from error
    if not isinstance(value, dict):
        raise ContractError(f"{path} must contain a JSON object")
    return value


class TrainedModelFolder:
    """An upstream trained model folder and the facts conversion and caching need about it."""

    def __init__(self, path: str | Path, checkpoint_name: str = UPSTREAM_CHECKPOINT) -> None:
        if Path(checkpoint_name).name != checkpoint_name:
            raise ContractError("checkpoint name must be a file name")
        self.path = Path(path)
        self.checkpoint_name = checkpoint_name

    def folds(self) -> tuple[int | str, ...]:
        """Folds with a checkpoint: numeric folds ascending, then ``"all"``."""
        found = []
        if self.path.is_dir():
            for entry in self.path.iterdir():
                fold = _fold_from_directory(entry.name)
                if fold is not None and (entry / self.checkpoint_name).is_file():
                    found.append(fold)
        if not found:
            raise ContractError(f"{self.path} has no fold_<n> (or fold_all) folder with a {self.checkpoint_name}")
        return tuple(sorted(found, key=_fold_order))

    def checkpoint(self, fold: int | str) -> Path:
        return self.path / f"fold_{fold}" / self.checkpoint_name

    def plans(self) -> dict:
        return _load_json_object(self.path / "plans.json")

    def dataset(self) -> dict:
        return _load_json_object(self.path / "dataset.json")

    def fingerprint(self, folds: Iterable[int | str]) -> dict:
        """Parsed plans and dataset plus (size, mtime) of every listed fold checkpoint."""
        checkpoints = {}
        for fold in folds:
            info = self.checkpoint(fold).stat()
            checkpoints[str(fold)] = [info.st_size, info.st_mtime_ns]
        return {"plans": self.plans(), "dataset": self.dataset(), "checkpoint_name": self.checkpoint_name,
                "checkpoints": checkpoints}


def detect_upstream_folds(model_folder: str | Path, *,
                          checkpoint_name: str = UPSTREAM_CHECKPOINT) -> tuple[int | str, ...]:
    """Numeric folds (ascending), then ``"all"``, whose ``fold_*`` folder holds ``checkpoint_name``."""
    return TrainedModelFolder(model_folder, checkpoint_name).folds()


def _normalise_folds(folds) -> tuple[int | str, ...]:
    chosen: list[int | str] = []
    for fold in folds:
        if isinstance(fold, str):
            parsed = _fold_from_directory(f"fold_{fold}")
        elif isinstance(fold, (int, np.integer)) and not isinstance(fold, bool) and fold >= 0:
            parsed = int(fold)
        else:
            parsed = None
        if parsed is None:
            raise ContractError(f"invalid fold {fold!r}")
        if parsed in chosen:
            raise ContractError(f"fold {parsed!r} is listed twice")
        chosen.append(parsed)
    if not chosen:
        raise ContractError("at least one fold is required")
    return tuple(chosen)


# ---------------------------------------------------------------------------- conversion
@dataclass(frozen=True, slots=True)
class ConversionResult:
    folder: Path
    configuration: str
    trainer_name: str
    folds: tuple[int | str, ...]


def _planned_spec(plans: dict, dataset_json: dict, configuration: str):
    from nnunet_mlx_b200.model.folder import _label_semantics, _spec_from_plans

    channels = dataset_json.get("channel_names") or dataset_json.get("modality")
    if not isinstance(channels, dict) or not channels:
        raise ContractError("dataset.json channel_names must be a non-empty mapping")
    output_channels, _ = _label_semantics(dataset_json)
    if configuration not in plans.get("configurations", {}):
        raise ContractError(f"plans.json has no configuration {configuration!r}")
    return _spec_from_plans(plans, configuration, len(channels), output_channels)


def _convert_fold(checkpoint: UpstreamCheckpoint, fold, spec, directory: Path) -> None:
    converted = convert_state_dict(checkpoint.network_weights)
    try:
        weights = validate_weights(spec, converted.weights)
    except ContractError as error:
        raise ContractError(f"fold {fold} weights do not match the network planned in plans.json: {error}") from error
    state = InferenceCheckpointState(
        identity=CheckpointIdentity(checkpoint.trainer_name, checkpoint.configuration, fold),
        current_epoch=checkpoint.current_epoch, spatial_dims=spec.spatial_dims,
        inference_allowed_mirroring_axes=checkpoint.mirroring_axes, dropped_source_keys=converted.dropped_keys)
    save_inference_checkpoint(directory, weights=weights, state=state)


def _verify_written(folder: Path, spec, configuration: str, folds) -> None:
    for fold in folds:
        directory = folder / f"fold_{fold}" / CONVERTED_CHECKPOINT
        identity = read_state(directory).identity
        if (identity.fold, identity.configuration) != (fold, configuration):
            raise ContractError(f"converted fold {fold} reads back as fold {identity.fold!r} / "
                                f"{identity.configuration!r}")
        validate_weights(spec, read_weights(directory))


def convert_trained_model(source: str | Path, destination: str | Path, *, folds: Sequence[int | str] | None = None,
                          checkpoint_name: str = UPSTREAM_CHECKPOINT) -> ConversionResult:
    """Convert a trained upstream model folder into a new converted model folder at ``destination``.

    All selected folds must share one plans-built trainer and one configuration
    and map exactly onto the network ``plans.json`` describes.  Nothing appears
    at ``destination`` (which must not exist yet) unless every fold converted
    and read back.
    """
    trained = TrainedModelFolder(source, checkpoint_name)
    if not trained.path.is_dir():
        raise ContractError(f"trained model folder does not exist: {trained.path}")
    target = Path(destination)
    if target.exists():
        raise ContractError(f"conversion destination exists: {target}")
    selected = trained.folds() if folds is None else _normalise_folds(folds)
    fingerprint = trained.fingerprint(selected)
    checkpoints = {fold: load_upstream_checkpoint(trained.checkpoint(fold)) for fold in selected}
    lead = checkpoints[selected[0]]
    if lead.trainer_name not in PLANS_BUILT_TRAINERS:
        raise ContractError(f"trainer {lead.trainer_name!r} is not supported: its network may differ from the one "
                            "plans.json describes")
    for fold, checkpoint in checkpoints.items():
        if (checkpoint.trainer_name, checkpoint.configuration) != (lead.trainer_name, lead.configuration):
            raise ContractError(f"fold {fold} was trained as {checkpoint.trainer_name}/{checkpoint.configuration}, "
                                f"fold {selected[0]} as {lead.trainer_name}/{lead.configuration}")
    spec = _planned_spec(fingerprint["plans"], fingerprint["dataset"], lead.configuration)
    target.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{target.name}.staging.", dir=target.parent))
    try:
        for name in ("plans.json", "dataset.json"):
            shutil.copyfile(trained.path / name, staging / name)
        for fold in selected:
            _convert_fold(checkpoints[fold], fold, spec, staging / f"fold_{fold}" / CONVERTED_CHECKPOINT)
        manifest = {
            "schema_version": CONVERSION_SCHEMA, "conversion_contract_version": CONVERSION_CONTRACT_VERSION,
            "source_folder": str(trained.path.absolute()), "source_fingerprint": fingerprint,
            "source_plans": fingerprint["plans"], "source_dataset": fingerprint["dataset"],
            "configuration": lead.configuration, "trainer_name": lead.trainer_name,
            "architecture": type(spec).__name__, "spatial_dims": spec.spatial_dims,
            "folds": [{"fold": fold, "checkpoint": CONVERTED_CHECKPOINT, "source_checkpoint": checkpoint_name}
                      for fold in selected],
        }
        (staging / CONVERSION_FILENAME).write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n",
                                                   encoding="utf-8")
        _verify_written(staging, spec, lead.configuration, selected)
        os.replace(staging, target)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise
    return ConversionResult(target, lead.configuration, lead.trainer_name, selected)


def read_conversion_manifest(folder: str | Path) -> dict:
    manifest = _load_json_object(Path(folder) / CONVERSION_FILENAME)
    if manifest.get("schema_version") != CONVERSION_SCHEMA:
        raise ContractError(f"{folder} was not written by this conversion (schema "
                            f"{manifest.get('schema_version')!r})")
    if not isinstance(manifest.get("configuration"), str) or not isinstance(manifest.get("folds"), list):
        raise ContractError(f"{folder}: the conversion manifest lacks its configuration or fold list")
    return manifest


# ---------------------------------------------------------------------------- results folder and cache
def _dataset_directory(root: Path, dataset: str) -> str:
    """A dataset name, or the one ``DatasetNNN_*`` directory of a numeric ID under ``root``."""
    if not dataset.isdigit():
        return dataset
    prefix = f"Dataset{int(dataset):03d}_"
    candidates = sorted(entry.name for entry in root.iterdir()
                        if entry.is_dir() and entry.name.startswith(prefix) and len(entry.name) > len(prefix)) \
        if root.is_dir() else []
    if len(candidates) != 1:
        found = ", ".join(candidates) if candidates else "none"
        raise ContractError(f"dataset {dataset} must match exactly one {prefix}* folder in {root} (found {found})")
    return candidates[0]


def resolve_results_folder(dataset: str, *, configuration: str, trainer: str = "nnUNetTrainer",
                           plans: str = "nnUNetPlans", results: str | Path | None = None) -> Path:
    """``<results>/<dataset>/<trainer>__<plans>__<configuration>`` as nnU-Net lays it out; ``dataset``
    is an ID (``3`` -> the one ``Dataset003_*`` folder) or a full name; ``results`` defaults to
    ``$nnUNet_results``."""
    location = results if results is not None else os.environ.get(RESULTS_VARIABLE)
    if not location:
        raise ContractError(f"no results folder: pass one, set ${RESULTS_VARIABLE}, or give a trained model "
                            "folder with -m")
    root = Path(location).expanduser()
    folder = root / _dataset_directory(root, str(dataset)) / f"{trainer}__{plans}__{configuration}"
    if not folder.is_dir():
        raise ContractError(f"trained model folder does not exist: {folder}")
    return folder


def _cache_entry(cache_root: Path, trained: Path) -> Path:
    """``<cache>/converted/<dataset directory>/<model directory>`` of a trained folder."""
    parts = trained.parts
    if len(parts) < 3:
        raise ContractError(f"{trained} needs a dataset directory and a model directory to be cached")
    return cache_root / "converted" / parts[-2] / parts[-1]


def _entry_is_current(entry: Path, trained: TrainedModelFolder, folds) -> bool:
    """Whether ``entry`` is a complete conversion of ``trained``'s current state for ``folds``."""
    try:
        manifest = read_conversion_manifest(entry)
        current = trained.fingerprint(folds)
    except (ContractError, OSError):
        return False
    if manifest.get("conversion_contract_version") != CONVERSION_CONTRACT_VERSION:
        return False
    if manifest.get("source_folder") != str(trained.path) or manifest.get("source_fingerprint") != current:
        return False
    return all((entry / f"fold_{fold}" / CONVERTED_CHECKPOINT / "weights.safetensors").is_file() for fold in folds)


def cached_conversion(trained_folder: str | Path, *, folds: Sequence[int | str] | None = None,
                      checkpoint_name: str = UPSTREAM_CHECKPOINT, cache: str | Path | None = None) -> Path:
    """A converted copy of ``trained_folder`` in the conversion cache (``cache``, else
    ``$NNUNET_MLX_CACHE``, else ``~/.cache/nnunet-mlx``) at ``converted/<dataset>/<model>``.

    Every available fold is converted; ``folds`` only states which must exist.
    The entry is rebuilt when the source plans, dataset or any fold checkpoint
    (size, modification time) differs from what it was converted from.
    """
    trained = TrainedModelFolder(Path(os.path.abspath(trained_folder)), checkpoint_name)
    available = trained.folds()
    if folds is not None:
        absent = [fold for fold in _normalise_folds(folds) if fold not in available]
        if absent:
            raise ContractError(f"folds {absent} have no {checkpoint_name} in {trained.path}")
    root = Path(cache if cache is not None else os.environ.get(CACHE_VARIABLE, DEFAULT_CACHE)).expanduser()
    entry = _cache_entry(root, trained.path)
    if entry.is_symlink():
        raise ContractError(f"refusing a symlinked conversion cache entry: {entry}")
    if _entry_is_current(entry, trained, available):
        return entry
    # complete the new conversion beside the old entry, then swap it in
    fresh = entry.with_name(f"{entry.name}.new")
    if fresh.exists():
        shutil.rmtree(fresh)
    convert_trained_model(trained.path, fresh, folds=available, checkpoint_name=checkpoint_name)
    if entry.exists():
        retired = entry.with_name(f"{entry.name}.old")
        shutil.rmtree(retired, ignore_errors=True)
        os.replace(entry, retired)
        os.replace(fresh, entry)
        shutil.rmtree(retired, ignore_errors=True)
    else:
        os.replace(fresh, entry)
    return entry
