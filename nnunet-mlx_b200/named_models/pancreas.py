"""``pancreas`` runner (reference ``src/nnunet_mlx/named_models/pancreas.py``): ``run`` and ``load_model``."""

from nnunet_mlx_b200.named_models import make

run, load_model = make("pancreas")

__all__ = ["load_model", "run"]
