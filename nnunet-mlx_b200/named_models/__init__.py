"""Released-model wrappers (reference ``src/nnunet_mlx/named_models``).

Each module exposes ``run`` and ``load_model`` with the reference's argument
names.  Weight download is outside this package: ``weights_path`` must point
at a local converted model folder.
"""

from __future__ import annotations

from nnunet_mlx_b200 import medmlx
from nnunet_mlx_b200.errors import ContractError

_CONFIGURATIONS = {
    "liver": ("nnunet-liver", "3d_fullres", None),
    "pancreas": ("nnunet-pancreas", "3d_fullres", None),
    "brats": ("nnunet-brats2021", "3d_fullres", None),
    "autopet": ("nnunet-autopet", "3d_fullres", None),
    "siam": ("siam", "3d_fullres", None),
    "mrsegmentator": ("mrsegmentator", "3d_fullres", None),
}


def _folder(name: str, weights_path):
    if weights_path is None:
        raise ContractError(f"{_CONFIGURATIONS[name][0]}: pass weights_path (a local converted model folder); "
                            "downloading released weights is not part of the B200 inference path")
    return weights_path


def make(name: str):
    repo, configuration, folds = _CONFIGURATIONS[name]

    def run(*, image_path, output_dir, weights_path=None, overwrite: bool = False, use_mirroring: bool = True,
            step_fraction: float = 0.5, precision: str = "native"):
        return medmlx.run(weights_path=_folder(name, weights_path), image_paths=[image_path], output_dir=output_dir,
                          overwrite=overwrite, configuration=configuration, folds=folds, precision=precision,
                          step_fraction=step_fraction, use_mirroring=use_mirroring)

    def load_model(*, weights_path=None, use_mirroring: bool = True, step_fraction: float = 0.5,
                   precision: str = "native"):
        return medmlx.load_model(weights_path=_folder(name, weights_path), configuration=configuration, folds=folds,
                                 precision=precision, step_fraction=step_fraction, use_mirroring=use_mirroring)

    run.__doc__ = f"Segment one preprocessed case with the {repo} model folder."
    load_model.__doc__ = f"Load the {repo} model folder once for several cases."
    return run, load_model
