"""Converted inference checkpoints: ``state.json`` + ``weights.safetensors``.

Reads and writes the directory format of reference
``src/nnunet_mlx/storage/checkpoint.py`` (schema constants 27-31,
``InferenceCheckpointState`` 54-113, ``load_inference_checkpoint`` 130-165,
exact file set 206-216), so converted model folders are interchangeable.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from nnunet_mlx_b200.errors import ContractError

SCHEMA_VERSION = "nnunet-mlx.checkpoint.v2"
INFERENCE_SCHEMA_VERSION = "nnunet-mlx.inference-checkpoint.v2"
SOURCE_NNUNET_VERSION = "v2.8.1"
_INFERENCE_FILES = {"weights.safetensors", "state.json"}
_TRAINING_FILES = {"weights.safetensors", "optimizer.safetensors", "rng.safetensors", "state.json"}


@dataclass(frozen=True, slots=True)
class CheckpointIdentity:
    trainer_name: str
    configuration: str
    fold: int | str

    def __post_init__(self) -> None:
        if not self.trainer_name or not self.configuration:
            raise ContractError("checkpoint trainer and configuration must be non-empty")
        if not ((isinstance(self.fold, int) and not isinstance(self.fold, bool) and self.fold >= 0)
                or self.fold == "all"):
            raise ContractError("checkpoint fold must be a non-negative integer or 'all'")


@dataclass(frozen=True, slots=True)
class InferenceCheckpointState:
    identity: CheckpointIdentity
    current_epoch: int | None
    spatial_dims: int
    inference_allowed_mirroring_axes: tuple[int, ...]
    dropped_source_keys: tuple[str, ...] = ()

    def __post_init__(self) -> None:
        axes = self.inference_allowed_mirroring_axes
        if self.spatial_dims not in (2, 3):
            raise ContractError("checkpoint spatial dimensions must be 2 or 3")
        if len(set(axes)) != len(axes) or any(a not in range(self.spatial_dims) for a in axes):
            raise ContractError(f"invalid checkpoint mirroring axes {axes}")

    def to_payload(self) -> dict[str, object]:
        return {
            "schema_version": INFERENCE_SCHEMA_VERSION,
            "source_nnunet_version": SOURCE_NNUNET_VERSION,
            "identity": {"trainer_name": self.identity.trainer_name,
                         "configuration": self.identity.configuration,
                         "fold": self.identity.fold},
            "current_epoch": self.current_epoch,
            "spatial_dims": self.spatial_dims,
            "inference_allowed_mirroring_axes": list(self.inference_allowed_mirroring_axes),
            "dropped_source_keys": list(self.dropped_source_keys),
        }


def _identity(value: object) -> CheckpointIdentity:
    if not isinstance(value, dict):
        raise ContractError("checkpoint identity must be a mapping")
    fold = value.get("fold")
    return CheckpointIdentity(str(value.get("trainer_name") or ""), str(value.get("configuration") or ""),
                              fold if fold == "all" else int(fold))


def read_state(directory: Path) -> InferenceCheckpointState:
    if not directory.is_dir():
        raise ContractError(f"checkpoint directory does not exist: {directory}")
    state_file = directory / "state.json"
    if not state_file.is_file():
        raise ContractError("checkpoint state.json does not exist")
    try:
        payload = json.loads(state_file.read_text(encoding="utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as error:
        raise ContractError("checkpoint state is invalid JSON") from error
    schema = payload.get("schema_version")
    names = {p.name for p in directory.iterdir()}
    if schema == INFERENCE_SCHEMA_VERSION:
        expected = _INFERENCE_FILES
    elif schema == SCHEMA_VERSION:
        expected = _TRAINING_FILES
    else:
        raise ContractError(f"unsupported inference checkpoint schema {schema!r}")
    if names != expected:
        raise ContractError(f"checkpoint file set mismatch: expected {sorted(expected)}, found {sorted(names)}")
    if payload.get("source_nnunet_version") != SOURCE_NNUNET_VERSION:
        raise ContractError("inference checkpoint source nnU-Net version does not match")
    epoch = payload.get("current_epoch")
    return InferenceCheckpointState(
        identity=_identity(payload.get("identity")),
        current_epoch=None if epoch is None else int(epoch),
        spatial_dims=int(payload.get("spatial_dims")),
        inference_allowed_mirroring_axes=tuple(int(a) for a in payload.get("inference_allowed_mirroring_axes", [])),
        dropped_source_keys=tuple(payload.get("dropped_source_keys", ()))
        if schema == INFERENCE_SCHEMA_VERSION else (),
    )


def read_weights(directory: Path) -> dict[str, np.ndarray]:
    from safetensors.numpy import load_file

    path = directory / "weights.safetensors"
    if not path.is_file():
        raise ContractError(f"checkpoint weights are unavailable: {path}")
    return {k: np.asarray(v, dtype=np.float32) for k, v in load_file(str(path)).items()}


def load_inference_checkpoint(directory: str | Path):
    """Return ``(state, weights)`` after checking the file set, schema and finiteness."""
    source = Path(directory)
    state = read_state(source)
    weights = read_weights(source)
    for key, value in weights.items():
        if not np.isfinite(value).all():
            raise ContractError(f"model tensor {key!r} is non-finite")
    return state, weights


def save_inference_checkpoint(directory: str | Path, *, weights: dict[str, np.ndarray],
                              state: InferenceCheckpointState) -> None:
    from safetensors.numpy import save_file

    target = Path(directory)
    if target.exists():
        raise ContractError(f"checkpoint directory already exists: {target}")
    target.mkdir(parents=True)
    save_file({k: np.ascontiguousarray(v, dtype=np.float32) for k, v in weights.items()},
              str(target / "weights.safetensors"))
    (target / "state.json").write_text(json.dumps(state.to_payload(), indent=2, sort_keys=True) + "\n",
                                       encoding="utf-8")


def weights_signature(directory: str | Path) -> list[int]:
    stat = (Path(directory) / "weights.safetensors").stat()
    return [stat.st_size, stat.st_mtime_ns]
