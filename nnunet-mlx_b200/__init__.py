"""B200-native inference path of nnunet-mlx: 3-D U-Net forward + Gaussian sliding window.

Public names follow reference ``src/nnunet_mlx/__init__.py:26-39``.
"""

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.topology import PlainConvUNetSpec, ResidualEncoderUNetSpec

__version__ = "0.1.0"

__all__ = [
    "ArrayPredictor",
    "ContractError",
    "ModelFolderPredictor",
    "NnUNetModel",
    "PlainConvUNetSpec",
    "ResidualEncoderUNetSpec",
    "load_model",
    "load_model_bundle",
    "run",
]


def __getattr__(name):
    # lazy imports keep `import nnunet_mlx_b200` free of torch/CUDA initialisation
    if name == "ArrayPredictor":
        from nnunet_mlx_b200.prediction.inference import ArrayPredictor
        return ArrayPredictor
    if name == "ModelFolderPredictor":
        from nnunet_mlx_b200.prediction.pipeline import ModelFolderPredictor
        return ModelFolderPredictor
    if name == "load_model_bundle":
        from nnunet_mlx_b200.model.folder import load_model_bundle
        return load_model_bundle
    if name in ("NnUNetModel", "load_model", "run"):
        from nnunet_mlx_b200 import medmlx
        return getattr(medmlx, name)
    raise AttributeError(name)
