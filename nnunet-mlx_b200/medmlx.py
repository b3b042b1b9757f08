"""Runner API: ``run``, ``load_model`` and ``NnUNetModel`` over a converted model folder.

Same entry-point names and core arguments as reference
``src/nnunet_mlx/medmlx.py`` (``run`` 203-278, ``NnUNetModel`` 486-587,
``load_model`` 590-605).  Inputs here are preprocessed ``(C, *spatial)``
float32 arrays or ``.npy`` / ``.npz`` files (NIfTI reading, preprocessing and
grid restoration are outside this package); outputs are written by
``ModelFolderPredictor.predict_case``.  ``precision`` selects the convolution
arithmetic: ``"fp32"`` (default: fp16 hi/lo operand pairs on the tensor cores,
three products and float32 accumulation, float32-level accuracy; volumes whose
activations leave the fp16 range are recomputed in split TF32) or ``"tf32"``
(single-pass, faster, looser).  The reference's ``"native"`` maps to
``"fp32"``.
"""

from __future__ import annotations

from dataclasses import replace
from pathlib import Path

from nnunet_mlx_b200.errors import ContractError

_PRECISIONS = {"native": "fp32", "fp32": "fp32", "tf32": "tf32"}

# Runner windows and folds accumulate in float16 as upstream nnU-Net does (reference medmlx.py:41-42,
# 121-134); ModelFolderPredictor's own float32 default is for direct Python use.
ACCUMULATION = "nnunet-fp16"


class NnUNetModel:
    """One loaded model folder reused for serial cases until closed."""

    def __init__(self, *, weights_path, configuration: str = "3d_fullres", folds=None,
                 checkpoint_name: str = "checkpoint_final", precision: str = "native",
                 step_fraction: float = 0.5, use_mirroring: bool = True, device="cuda") -> None:
        from nnunet_mlx_b200.model.folder import load_model_bundle
        from nnunet_mlx_b200.prediction.pipeline import ModelFolderPredictor

        if precision not in _PRECISIONS:
            raise ContractError(f"unsupported precision {precision!r}")
        if not isinstance(use_mirroring, bool):
            raise ContractError("use_mirroring must be a boolean")
        if not 0 < float(step_fraction) <= 1:
            raise ContractError("step_fraction must be in (0, 1]")
        if Path(checkpoint_name).name != checkpoint_name or checkpoint_name in {".", ".."}:
            raise ContractError("checkpoint_name must name a checkpoint directory")
        bundle = load_model_bundle(Path(weights_path).expanduser(), configuration=configuration, folds=folds,
                                   checkpoint_name=checkpoint_name, precision=_PRECISIONS[precision],
                                   device=device)
        if not use_mirroring:
            bundle = replace(bundle, mirroring_axes=())
        self._predictor: ModelFolderPredictor | None = ModelFolderPredictor(
            bundle, step_fraction=step_fraction, accumulation=ACCUMULATION)

    def run(self, *, image_paths, output_dir, overwrite: bool = False, save_probabilities: bool = False) -> dict:
        if self._predictor is None:
            raise RuntimeError("nnU-Net model is closed")
        images = [Path(p) for p in image_paths]
        if len(images) != 1:
            raise ContractError("pass one preprocessed (C, *spatial) array file per case")
        out_dir = Path(output_dir)
        prefix = out_dir / images[0].stem
        if Path(f"{prefix}.npz").exists() and not overwrite:
            raise ContractError(f"output exists: {prefix}.npz (pass overwrite=True)")
        return self._predictor.predict_case(images, prefix, save_probabilities=save_probabilities)

    def segment_array(self, data, *, return_probabilities: bool = False):
        if self._predictor is None:
            raise RuntimeError("nnU-Net model is closed")
        return self._predictor.predict_preprocessed(data, return_probabilities=return_probabilities)

    def close(self) -> None:
        self._predictor = None

    def __enter__(self) -> "NnUNetModel":
        return self

    def __exit__(self, *args) -> None:
        self.close()


def load_model(*, weights_path, configuration: str = "3d_fullres", folds=None,
               checkpoint_name: str = "checkpoint_final", precision: str = "native", step_fraction: float = 0.5,
               use_mirroring: bool = True) -> NnUNetModel:
    """Load a model folder once for several cases (reference ``load_model`` 590-605)."""
    return NnUNetModel(weights_path=weights_path, configuration=configuration, folds=folds,
                       checkpoint_name=checkpoint_name, precision=precision, step_fraction=step_fraction,
                       use_mirroring=use_mirroring)


def run(*, weights_path, image_paths, output_dir, overwrite: bool = False, configuration: str | None = None,
        folds=None, checkpoint_name: str = "checkpoint_final", precision: str = "native",
        step_fraction: float = 0.5, use_mirroring: bool = True, save_probabilities: bool = False) -> dict:
    """Segment one case with a local converted model folder (reference ``run`` 203-278)."""
    with NnUNetModel(weights_path=weights_path, configuration=configuration or "3d_fullres", folds=folds,
                     checkpoint_name=checkpoint_name, precision=precision, step_fraction=step_fraction,
                     use_mirroring=use_mirroring) as model:
        return model.run(image_paths=image_paths, output_dir=output_dir, overwrite=overwrite,
                         save_probabilities=save_probabilities)
