"""``brats`` runner (reference ``src/nnunet_mlx/named_models/brats.py``): ``run`` and ``load_model``."""

from nnunet_mlx_b200.named_models import make

run, load_model = make("brats")

__all__ = ["load_model", "run"]
