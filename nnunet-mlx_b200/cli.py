"""``nnunet-mlx predict``-compatible command line for the B200 path.

Option names follow reference ``src/nnunet_mlx/commands/upstream.py:56-118``
(nnUNetv2_predict's flags).  Inputs are preprocessed ``(C, *spatial)``
``.npy`` / ``.npz`` cases in the ``-i`` folder.  The model is ``-m`` (a
converted model folder, or a trained upstream folder with
``fold_*/checkpoint_final.pth``) or ``-d DATASET [-tr TRAINER] [-p PLANS]``
resolved under ``$nnUNet_results``; upstream folders are converted once into
the conversion cache (``storage.upstream.cached_conversion``).  Flags that only concern raw-image I/O or the reference's process
pools (``-npp``, ``-nps``, ``-prev_stage_predictions``, ``--max-inflight-bytes``)
are accepted and ignored.

    python -m nnunet_mlx_b200.cli predict -i IN -o OUT (-m MODEL | -d DATASET [-tr T] [-p P]) [-f 0 1 ...]
        [--disable_tta] [--save_probabilities] [--continue_prediction] [-num_parts N -part_id K]
        [-c 3d_fullres] [-chk checkpoint_final] [--precision fp32|tf32] [--json]
"""

from __future__ import annotations

import argparse
import json
import sys
from dataclasses import replace
from pathlib import Path

from nnunet_mlx_b200.errors import ContractError


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="nnunet-mlx")
    sub = parser.add_subparsers(dest="command", required=True)
    p = sub.add_parser("predict", help="predict a folder of preprocessed cases")
    p.add_argument("-i", dest="input_folder", required=True)
    p.add_argument("-o", dest="output_folder", required=True)
    p.add_argument("-m", dest="model_folder", default=None)
    p.add_argument("-d", dest="dataset", default=None)
    p.add_argument("-tr", dest="trainer", default="nnUNetTrainer")
    p.add_argument("-p", dest="plans", default="nnUNetPlans")
    p.add_argument("-c", dest="configuration", default="3d_fullres")
    p.add_argument("-f", dest="folds", nargs="+", default=None)
    p.add_argument("-chk", dest="checkpoint_name", default="checkpoint_final")
    p.add_argument("-step_size", dest="step_size", type=float, default=0.5)
    p.add_argument("--disable_tta", action="store_true")
    p.add_argument("--save_probabilities", action="store_true")
    p.add_argument("--continue_prediction", action="store_true")
    p.add_argument("-num_parts", type=int, default=1)
    p.add_argument("-part_id", type=int, default=0)
    p.add_argument("-npp", type=int, default=0)
    p.add_argument("-nps", type=int, default=0)
    p.add_argument("-prev_stage_predictions", default=None)
    p.add_argument("--max-inflight-bytes", type=int, default=2 * 1024**3)
    p.add_argument("--precision", choices=["fp32", "tf32"], default="fp32")
    p.add_argument("--json", dest="json_output", action="store_true")
    return parser


def resolve_model(args, folds) -> tuple[Path, str]:
    """(converted model folder, checkpoint directory name) for ``-m`` or ``-d``; trained upstream
    folders (``fold_*/<checkpoint>.pth``) go through the conversion cache."""
    from nnunet_mlx_b200.storage.upstream import CONVERTED_CHECKPOINT, cached_conversion, resolve_results_folder

    if (args.model_folder is None) == (args.dataset is None):
        raise ContractError("pass exactly one of -m MODEL_FOLDER and -d DATASET")
    folder = Path(args.model_folder) if args.model_folder is not None else resolve_results_folder(
        args.dataset, configuration=args.configuration, trainer=args.trainer, plans=args.plans)
    name = args.checkpoint_name.removesuffix(".pth")
    if any(folder.glob(f"fold_*/{name}.pth")):
        return cached_conversion(folder, folds=folds, checkpoint_name=f"{name}.pth"), CONVERTED_CHECKPOINT
    return folder, name


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    try:
        if not 0 < args.step_size <= 1:
            raise ContractError("-step_size must be in (0, 1]")
        if args.prev_stage_predictions is not None:
            raise ContractError("cascade (-prev_stage_predictions) inputs are not supported")
        from nnunet_mlx_b200.model.folder import load_model_bundle
        from nnunet_mlx_b200.prediction.pipeline import ModelFolderPredictor

        folds = None if args.folds is None else [f if f == "all" else int(f) for f in args.folds]
        model_folder, checkpoint_name = resolve_model(args, folds)
        bundle = load_model_bundle(model_folder, configuration=args.configuration, folds=folds,
                                   checkpoint_name=checkpoint_name, precision=args.precision)
        if args.disable_tta:
            bundle = replace(bundle, mirroring_axes=())
        from nnunet_mlx_b200.medmlx import ACCUMULATION

        # the predict command accumulates in float16 like upstream (reference commands/upstream.py:161-162)
        predictor = ModelFolderPredictor(bundle, step_fraction=args.step_size, accumulation=ACCUMULATION)
        results = predictor.predict_folder(args.input_folder, args.output_folder,
                                           save_probabilities=args.save_probabilities,
                                           continue_prediction=args.continue_prediction,
                                           num_parts=args.num_parts, part_id=args.part_id)
        if args.json_output:
            print(json.dumps({"status": "ok", "cases": results}))
        return 0
    except ContractError as error:
        print(json.dumps({"status": "error", "error": str(error)}), file=sys.stderr)
        return 2


if __name__ == "__main__":
    sys.exit(main())
