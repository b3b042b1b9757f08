"""``ModelFolderPredictor``: the case-level caller of the inference path.

Keeps the constructor and the ``self.predictor`` seam of reference
``src/nnunet_mlx/prediction/pipeline.py:171-215`` (an ``ArrayPredictor`` over
the bundle's fold models).  Image-file I/O and export are outside this
package's scope.  Cases are passed either raw, as ``(C, X, Y, Z)`` arrays with
their spacing (``predict_raw_case``: device preprocessing, inference and
restoration), or preprocessed, as ``(C, *spatial)`` float32 arrays in memory or
``.npy`` / ``.npz`` files, written as ``.npz`` (labels, optional
probabilities/logits).
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.folder import ModelBundle
from nnunet_mlx_b200.prediction.inference import (
    ArrayPredictor,
    logits_to_probabilities,
    probabilities_to_segmentation,
)


@dataclass(frozen=True)
class PredictionMetrics:
    """Timings of one case (reference ``PredictionMetrics`` pipeline.py:56-79)."""

    tile_inference_s: float
    total_s: float
    tiles: int
    shape: tuple[int, ...]
    patch_size: tuple[int, ...]

    def to_payload(self) -> dict[str, object]:
        return {"tile_inference_s": self.tile_inference_s, "total_s": self.total_s, "tiles": self.tiles,
                "shape": list(self.shape), "patch_size": list(self.patch_size)}


def _load_case(path: Path) -> np.ndarray:
    if path.suffix == ".npy":
        data = np.load(path)
    elif path.suffix == ".npz":
        with np.load(path) as z:
            data = z["data"] if "data" in z.files else z[z.files[0]]
    else:
        raise ContractError(f"unsupported case file {path.name}: expected preprocessed .npy/.npz")
    return np.ascontiguousarray(data, dtype=np.float32)


class ModelFolderPredictor:
    """Predict cases with a loaded model bundle on one B200."""

    def __init__(self, bundle: ModelBundle, *, step_fraction: float = 0.5, compile_models: bool = False,
                 accumulation: str = "float32") -> None:
        if compile_models:
            raise ContractError("compile_models is an MLX option; the B200 path runs pre-built CUDA kernels")
        self.bundle = bundle
        self.predictor = ArrayPredictor(
            bundle.models, patch_size=bundle.patch_size, num_outputs=bundle.output_channels,
            mirroring_axes=bundle.mirroring_axes, regions_class_order=bundle.regions_class_order,
            step_fraction=step_fraction, accumulation=accumulation)
        self.step_fraction = step_fraction

    def predict_preprocessed(self, data: np.ndarray, *, return_probabilities: bool = False):
        """Labels (uint16) and optionally probabilities for one preprocessed case."""
        from nnunet_mlx_b200.prediction.sliding_window import volume_work

        data = np.ascontiguousarray(data, dtype=np.float32)
        if data.ndim != 4 or data.shape[0] != self.bundle.image_channels:
            raise ContractError(f"expected ({self.bundle.image_channels}, z, y, x) preprocessed data, "
                                f"got {data.shape}")
        start = time.perf_counter()
        regions = self.bundle.regions_class_order
        probabilities = None
        if return_probabilities or regions is not None:
            logits = self.predictor.predict_logits_from_preprocessed_data(data)
            probabilities = logits_to_probabilities(logits, has_regions=regions is not None)
            labels = probabilities_to_segmentation(probabilities, regions_class_order=regions)
        else:
            labels = self.predictor.predict_labels_from_preprocessed_data(data)
        elapsed = time.perf_counter() - start
        work = volume_work(data.shape[1:], self.bundle.patch_size, self.step_fraction,
                           2 ** len(self.bundle.mirroring_axes), len(self.bundle.models))
        metrics = PredictionMetrics(elapsed, elapsed, work["tiles"], tuple(data.shape[1:]), self.bundle.patch_size)
        return labels, probabilities, metrics

    def predict_raw_case(self, data, properties, *, device=None):
        """Raw case -> labels in the image's own grid and axis order, every step on the GPU.

        The reference's ``predict_case`` chain (``prediction/pipeline.py:257-387``: preprocess ->
        infer -> restore) without the file I/O: ``preprocess_raw_case`` (transpose, nonzero crop,
        normalisation, resampling to the plans' spacing) leaves the case on the device, the fold
        ensemble's sliding window reads it there, and the class logits are restored (resampled to
        the crop, first argmax, uncropped, transposed back) on the device; only the uint16 label
        volume crosses to the host.  ``data`` is ``(C, X, Y, Z)`` in the image's axis order,
        ``properties["spacing"]`` its voxel size.  Region models raise ``ContractError``.
        """
        from nnunet_mlx_b200.data.preprocessing import (
            PreprocessingPlans,
            ResamplingContract,
            preprocess_raw_case,
        )
        from nnunet_mlx_b200.prediction.restore import (
            LabelSemantics,
            plans_from_payload,
            restore_segmentation_on_device,
        )
        from nnunet_mlx_b200.prediction.sliding_window import volume_work

        if self.bundle.regions_class_order is not None:
            raise ContractError("region models are restored on the host (sigmoid probabilities)")
        plans = self.bundle.plans
        configuration = self.bundle.configuration
        config = plans.get("configurations", {}).get(configuration, {})
        start = time.perf_counter()
        prepared = preprocess_raw_case(data, properties,
                                       PreprocessingPlans.from_payload(plans, configuration=configuration),
                                       device=device)
        logits = self.predictor.predict_device_logits_from_preprocessed_data(prepared.data)
        restored = restore_segmentation_on_device(
            logits, prepared.properties, plans_from_payload(plans, configuration=configuration),
            LabelSemantics(self.bundle.output_channels),
            probability_resampling=ResamplingContract.from_configuration(
                config, field="resampling_fn_probabilities", expected_is_seg=False))
        elapsed = time.perf_counter() - start
        shape = tuple(int(v) for v in prepared.data.shape[1:])
        work = volume_work(shape, self.bundle.patch_size, self.step_fraction,
                           2 ** len(self.bundle.mirroring_axes), len(self.bundle.models))
        return restored.segmentation, prepared.properties, PredictionMetrics(elapsed, elapsed, work["tiles"], shape,
                                                                            self.bundle.patch_size)

    def predict_case(self, image_files, output_prefix, *, save_probabilities: bool = False):
        """Predict one preprocessed case file and write ``<output_prefix>.npz``."""
        files = [Path(f) for f in image_files]
        if len(files) != 1:
            raise ContractError("pass one preprocessed (C, *spatial) array file per case")
        labels, probabilities, metrics = self.predict_preprocessed(_load_case(files[0]),
                                                                   return_probabilities=save_probabilities)
        out = Path(f"{output_prefix}.npz")
        out.parent.mkdir(parents=True, exist_ok=True)
        payload = {"segmentation": labels}
        if save_probabilities and probabilities is not None:
            payload["probabilities"] = probabilities
        tmp = out.with_name(out.name + ".tmp.npz")
        np.savez_compressed(tmp, **payload)
        tmp.replace(out)
        return {"output": str(out), "metrics": metrics.to_payload()}

    def predict_folder(self, input_folder, output_folder, *, save_probabilities: bool = False,
                       continue_prediction: bool = False, num_parts: int = 1, part_id: int = 0):
        """Predict every ``.npy``/``.npz`` case of a folder; ``cases[part_id::num_parts]`` partitioning."""
        if not 0 <= part_id < num_parts:
            raise ContractError("part_id must be in [0, num_parts)")
        cases = sorted(p for p in Path(input_folder).iterdir() if p.suffix in (".npy", ".npz"))
        results = []
        for path in cases[part_id::num_parts]:
            prefix = Path(output_folder) / path.stem
            if continue_prediction and Path(f"{prefix}.npz").exists():
                continue
            results.append(self.predict_case([path], prefix, save_probabilities=save_probabilities))
        return results
