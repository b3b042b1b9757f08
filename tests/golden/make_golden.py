"""Generate the golden vectors under ``tests/golden`` from the reference's own code.

Run in a container where the reference checkout is available::

    python tests/golden/make_golden.py /path/to/nnunet-mlx

It imports only the reference's pure-host helpers, which run without MLX:

* ``nnunet_mlx.prediction.sliding_window.compute_steps`` (reference 32-67),
  ``gaussian_importance`` (70-93) and ``nnunet_fp16_gaussian`` (96-113);
* ``nnunet_mlx.storage.weights.map_key_and_layout`` / ``convert_state_dict``
  (reference 48-182) applied to upstream-style state-dict keys;
* ``nnunet_mlx.prediction.inference.logits_to_probabilities`` /
  ``probabilities_to_segmentation`` (reference 210-269);
* ``nnunet_mlx.kernels.metal_restore._axis_metadata`` (reference 476-495, the
  fused restoration's per-axis indices and double-single weights) and
  ``device_class_restore_supported`` (336-360), and
  ``nnunet_mlx.data.resampling.separate_z_axis`` (587-616).

It also copies the reference's recorded upstream vectors from
``tests/fixtures/darwin-arm64/upstream_runner.npz`` (head conversion arrays and
float16 fold-rounding probes) and from ``tests/fixtures/darwin-arm64/torch_resampling.npz``
(upstream ``resample_torch_fornnunet`` label resampling for every tie rule, mode and
separate-axis policy, and the cascade labels of twelve recorded ``preprocess_raw_case``
runs with their nonzero mask, previous-stage input, plans and geometry).  Outputs:
``geometry.json``, ``gaussian.npz``, ``weights_map.json``, ``upstream_runner_subset.npz``,
``restore_axes.npz``, ``restore_policy.json``, ``torch_resampling_labels.npz``,
``nearest_axis.json`` (``nnunet_mlx.data.resampling.nearest_axis_indices``, reference 401-407),
``preprocess_policy.json`` (``nnunet_mlx.plans.ResamplingContract.from_configuration`` on accepted and
rejected plan entries, ``nnunet_mlx.data.resampling.compute_new_shape``), and
``preprocess_reference.npz`` (the reference's own ``preprocess_raw_case``, reference
``data/preprocessing.py:60-163``, on grid-preserving plans: every normalisation scheme, masks
with holes, transposes, input dtypes, a cascade input), and ``plans_reference.json`` (the reference's
``PlansContract.from_payload`` view of every recorded plans payload plus three spline variants).  Nothing at
test time reads the reference checkout.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Geometry cases: the benchmark volumes (z padded to the patch where smaller),
# the reference tests' small shapes and odd edge cases.
STEP_CASES = [
    ((128, 128, 128), (128, 128, 128), 0.5),
    ((128, 768, 768), (128, 128, 128), 0.5),
    ((155, 240, 240), (128, 128, 128), 0.5),
    ((284, 400, 400), (128, 128, 128), 0.5),
    ((17, 33, 49), (16, 32, 32), 0.5),
    ((4, 4, 4), (4, 4, 4), 0.5),
    ((5, 6, 7), (4, 4, 4), 0.5),
    ((9, 10, 11), (4, 4, 4), 0.5),
    ((200, 123, 77), (64, 48, 32), 0.33),
    ((300, 300, 300), (96, 160, 160), 1.0),
    ((129, 130, 131), (128, 64, 32), 0.25),
    ((101, 257), (80, 96), 0.5),
]

GAUSSIAN_FULL = [(4, 4, 4), (5, 6, 7), (16, 32, 32), (4, 5), (7, 9)]
GAUSSIAN_SUMMARY = [(128, 128, 128), (96, 160, 160), (80, 192, 160)]
FP16_GAUSSIAN = [(4, 4, 4), (16, 32, 32), (8, 8, 8)]

# Restoration: (source, target) axis sizes (the reference tests' shapes, the
# benchmark grids, up/down by odd ratios, size-1 axes) ...
RESTORE_AXES = [(2, 3), (3, 5), (4, 7), (5, 3), (7, 4), (11, 6), (1, 3), (5, 7), (7, 1), (4, 7), (5, 8),
                (6, 9), (3, 3), (128, 128), (101, 128), (614, 768), (768, 614), (240, 155), (400, 401),
                (1, 1), (2, 1), (9, 2)]
# ... support decisions: (source, target, current spacing, new spacing,
# (function, order, order_z, force_separate_z, threshold), classes).
_ORDER1 = ("resample_data_or_seg_to_shape", 1, 0, False, 3.0)
_AUTO1 = ("resample_data_or_seg_to_shape", 1, 0, None, 3.0)
_ORDER3 = ("resample_data_or_seg_to_shape", 3, 0, None, 3.0)
_TORCH = ("resample_torch_fornnunet", 1, 0, None, 3.0)
RESTORE_SUPPORT = [
    ((4, 5, 6), (7, 8, 9), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER1, 3),
    ((4, 5, 6), (4, 5, 6), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER3, 3),
    ((4, 5, 6), (4, 5, 6), (5.0, 1.0, 1.0), (1.0, 1.0, 1.0), _TORCH, 3),
    ((4, 5, 6), (7, 8, 9), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER3, 3),
    ((4, 5, 6), (7, 8, 9), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0), _TORCH, 3),
    ((40, 50, 50), (120, 60, 60), (3.0, 0.8, 0.8), (1.0, 0.7, 0.7), _AUTO1, 3),
    ((40, 50, 50), (120, 60, 60), (2.5, 0.8, 0.8), (1.0, 0.7, 0.7), _AUTO1, 3),
    ((40, 50, 50), (120, 60, 60), (1.0, 1.0, 1.0), (4.0, 1.0, 1.0), _AUTO1, 3),
    ((40, 50, 50), (120, 60, 60), (1.0, 4.0, 4.0), (1.0, 1.0, 1.0), _AUTO1, 3),
    ((40, 50, 50), (120, 60, 60), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0),
     ("resample_data_or_seg_to_shape", 1, 0, True, 3.0), 3),
    ((40, 50, 50), (120, 60, 60), (2.0, 1.0, 1.0), (1.0, 1.0, 1.0),
     ("resample_data_or_seg_to_shape", 1, 0, True, 3.0), 3),
    ((40, 50, 50), (120, 60, 60), (2.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER1, 0),
    ((40, 50, 50), (120, 60, 60), (2.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER1, 65536),
    ((40, 50, 50), (120, 60, 60), (2.0, 1.0, 1.0), (1.0, 1.0, 1.0), _ORDER1, 65537),
    ((101, 768, 768), (101, 768, 768), (2.5, 0.8, 0.8), (2.5, 0.8, 0.8), _AUTO1, 3),
    ((101, 614, 614), (101, 768, 768), (2.5, 1.0, 1.0), (2.5, 0.8, 0.8), _AUTO1, 3),
    ((101, 614, 614), (101, 768, 768), (5.0, 1.0, 1.0), (5.0, 0.8, 0.8), _AUTO1, 3),
]
SEPARATE_Z = [((3.0, 0.8, 0.8), (1.0, 1.0, 1.0), None, 3.0), ((1.0, 1.0, 1.0), (1.0, 1.0, 3.5), None, 3.0),
              ((1.0, 1.0, 1.0), (3.5, 3.5, 1.0), None, 3.0), ((2.0, 1.0, 1.0), (1.0, 1.0, 1.0), True, 3.0),
              ((1.0, 1.0, 1.0), (1.0, 1.0, 1.0), True, 3.0), ((5.0, 1.0, 1.0), (1.0, 1.0, 1.0), False, 3.0),
              ((2.5, 0.8, 0.8), (2.5, 0.8, 0.8), None, 3.0), ((2.5, 0.8, 0.8), (2.5, 0.8, 0.8), None, 2.0)]


def _upstream_plain_keys(stages: int, enc_convs, dec_convs, cin, feats, classes, k=3):
    """Upstream dynamic-network-architectures PlainConvUNet state-dict shapes."""
    shapes: dict[str, tuple[int, ...]] = {}
    ch = cin
    for s in range(stages):
        for c in range(enc_convs[s]):
            ci = ch if c == 0 else feats[s]
            p = f"encoder.stages.{s}.0.convs.{c}"
            shapes[f"{p}.conv.weight"] = (feats[s], ci, k, k, k)
            shapes[f"{p}.conv.bias"] = (feats[s],)
            shapes[f"{p}.norm.weight"] = (feats[s],)
            shapes[f"{p}.norm.bias"] = (feats[s],)
            shapes[f"{p}.all_modules.0.weight"] = (feats[s], ci, k, k, k)
        ch = feats[s]
    for d in range(stages - 1):
        below, skip = feats[stages - 1 - d], feats[stages - 2 - d]
        shapes[f"decoder.transpconvs.{d}.weight"] = (below, skip, 2, 2, 2)
        shapes[f"decoder.transpconvs.{d}.bias"] = (skip,)
        for c in range(dec_convs[d]):
            ci = 2 * skip if c == 0 else skip
            p = f"decoder.stages.{d}.convs.{c}"
            shapes[f"{p}.conv.weight"] = (skip, ci, k, k, k)
            shapes[f"{p}.conv.bias"] = (skip,)
            shapes[f"{p}.norm.weight"] = (skip,)
            shapes[f"{p}.norm.bias"] = (skip,)
        shapes[f"decoder.seg_layers.{d}.weight"] = (classes, skip, 1, 1, 1)
        shapes[f"decoder.seg_layers.{d}.bias"] = (classes,)
        shapes[f"decoder.encoder.stages.0.0.convs.0.conv.weight"] = (feats[0], cin, k, k, k)
    return shapes


def _upstream_residual_keys(cin, feats, blocks, classes, k=3):
    shapes: dict[str, tuple[int, ...]] = {}
    stem = feats[0]
    shapes["encoder.stem.convs.0.conv.weight"] = (stem, cin, k, k, k)
    shapes["encoder.stem.convs.0.conv.bias"] = (stem,)
    shapes["encoder.stem.convs.0.norm.weight"] = (stem,)
    shapes["encoder.stem.convs.0.norm.bias"] = (stem,)
    ch = stem
    for s, f in enumerate(feats):
        for b in range(blocks[s]):
            ci = ch if b == 0 else f
            p = f"encoder.stages.{s}.blocks.{b}"
            shapes[f"{p}.conv1.conv.weight"] = (f, ci, k, k, k)
            shapes[f"{p}.conv1.conv.bias"] = (f,)
            shapes[f"{p}.conv1.norm.weight"] = (f,)
            shapes[f"{p}.conv1.norm.bias"] = (f,)
            shapes[f"{p}.conv2.conv.weight"] = (f, f, k, k, k)
            shapes[f"{p}.conv2.conv.bias"] = (f,)
            shapes[f"{p}.conv2.norm.weight"] = (f,)
            shapes[f"{p}.conv2.norm.bias"] = (f,)
            if b == 0 and ci != f:
                shapes[f"{p}.skip.1.conv.weight"] = (f, ci, 1, 1, 1)
                shapes[f"{p}.skip.1.norm.weight"] = (f,)
                shapes[f"{p}.skip.1.norm.bias"] = (f,)
        ch = f
    for d in range(len(feats) - 1):
        below, skip = feats[len(feats) - 1 - d], feats[len(feats) - 2 - d]
        shapes[f"decoder.transpconvs.{d}.weight"] = (below, skip, 2, 2, 2)
        shapes[f"decoder.transpconvs.{d}.bias"] = (skip,)
        p = f"decoder.stages.{d}.convs.0"
        shapes[f"{p}.conv.weight"] = (skip, 2 * skip, k, k, k)
        shapes[f"{p}.conv.bias"] = (skip,)
        shapes[f"{p}.norm.weight"] = (skip,)
        shapes[f"{p}.norm.bias"] = (skip,)
        shapes[f"decoder.seg_layers.{d}.weight"] = (classes, skip, 1, 1, 1)
        shapes[f"decoder.seg_layers.{d}.bias"] = (classes,)
    return shapes


class _Tensor:
    """Minimal object with the ``detach().cpu().numpy()`` chain the converter expects."""

    def __init__(self, array: np.ndarray) -> None:
        self.array = array

    def detach(self):
        return self

    def cpu(self):
        return self

    def numpy(self):
        return self.array


NEAREST_AXIS_CASES = [(1, 1), (1, 4), (3, 7), (7, 3), (5, 5), (10, 4), (4, 10), (101, 81), (81, 101), (2, 3),
                      (3, 2), (13, 26), (26, 13), (9, 14), (14, 9), (63, 64), (64, 63)]


_TORCH = "resample_torch_fornnunet"
_SPLINE = "resample_data_or_seg_to_shape"
PLAN_ENTRY_CASES = [
    (_TORCH, {"is_seg": False}, False), (_TORCH, {"is_seg": False, "mode": "nearest"}, False),
    (_TORCH, {"is_seg": False, "mode": "cubic"}, False), (_TORCH, {"is_seg": False, "aniso_axis_mode": "linear"}, False),
    (_TORCH, {"is_seg": False, "force_separate_z": True}, False),
    (_TORCH, {"is_seg": False, "force_separate_z": "yes"}, False),
    (_TORCH, {"is_seg": True, "seg_tiebreak": "lowest"}, True), (_TORCH, {"is_seg": True, "seg_tiebreak": "middle"}, True),
    (_TORCH, {"is_seg": False, "separate_z_anisotropy_threshold": 2}, False),
    (_TORCH, {"is_seg": False, "separate_z_anisotropy_threshold": 0}, False),
    (_TORCH, {"is_seg": False, "num_threads": 8}, False), (_TORCH, {"is_seg": False, "device": "cuda"}, False),
    (_TORCH, {"is_seg": False, "memefficient_seg_resampling": False}, False), (_TORCH, {"is_seg": False, "bogus": 1}, False),
    (_TORCH, {"is_seg": False, "order": 3}, False), (_TORCH, {"is_seg": True}, False), (_TORCH, {}, False),
    (_SPLINE, {"is_seg": False}, False), (_SPLINE, {"is_seg": False, "order": 1}, False),
    (_SPLINE, {"is_seg": False, "order": 6}, False), (_SPLINE, {"is_seg": False, "order": -1}, False),
    (_SPLINE, {"is_seg": False, "order_z": 3}, False), (_SPLINE, {"is_seg": False, "force_separate_z": None}, False),
    (_SPLINE, {"is_seg": False, "force_separate_z": True}, False),
    (_SPLINE, {"is_seg": True, "seg_tiebreak": "highest"}, True), (_SPLINE, {"is_seg": False, "num_threads": 2}, False),
    (_SPLINE, {"is_seg": False, "order": True}, False),
    (_SPLINE, {"is_seg": False, "separate_z_anisotropy_threshold": 1.5}, False),
    (_SPLINE, {"is_seg": False, "order": 3, "order_z": 0, "force_separate_z": None}, False),
    ("resample_with_magic", {"is_seg": False}, False),
]
NEW_SHAPE_CASES = [((5, 5, 5), (1.0, 1.0, 1.0), (2.0, 2.0, 2.0)), ((7, 4, 6), (5.0, 0.7, 1.6), (2.5, 1.4, 0.8)),
                   ((101, 768, 768), (5.0, 0.8, 0.8), (5.0, 1.0, 1.0)), ((3, 3, 3), (1.5, 1.5, 1.5), (1.0, 1.0, 1.0)),
                   ((155, 240, 240), (1.0, 1.0, 1.0), (1.0, 1.0, 1.0)), ((284, 400, 400), (3.0, 2.0364, 2.0364),
                                                                        (3.0, 2.0364, 2.0364)),
                   ((1, 9, 11), (999.0, 0.5, 0.5), (999.0, 0.75, 0.75)), ((33, 65), (0.6, 0.6), (0.9, 0.9))]


PREPROCESS_CASES = [
    ("ct-int16", np.int16, ("CTNormalization",), (False,), (0, 1, 2), False),
    ("ct-transposed", np.int16, ("CTNormalization",), (False,), (2, 0, 1), False),
    ("zscore-mask", np.float32, ("ZScoreNormalization",), (True,), (1, 2, 0), False),
    ("zscore-all", np.float64, ("ZScoreNormalization",), (False,), (0, 2, 1), False),
    ("rescale", np.int32, ("RescaleTo01Normalization",), (False,), (0, 1, 2), False),
    ("rgb", np.uint8, ("RGBTo01Normalization",), (False,), (2, 1, 0), False),
    ("none", np.float32, ("NoNormalization",), (False,), (0, 1, 2), False),
    ("mixed", np.float32, ("CTNormalization", "ZScoreNormalization", "RescaleTo01Normalization"),
     (False, True, False), (2, 0, 1), False),
    ("cascade", np.uint16, ("ZScoreNormalization",), (True,), (2, 0, 1), True),
]


def main(reference: Path) -> None:
    sys.path.insert(0, str(reference / "src"))
    from nnunet_mlx.prediction import inference
    from nnunet_mlx.prediction.sliding_window import (
        compute_steps,
        gaussian_importance,
        nnunet_fp16_gaussian,
    )
    from nnunet_mlx.storage.weights import convert_state_dict, map_key_and_layout

    geometry = [
        {"image": list(i), "patch": list(p), "step": s,
         "steps": [list(a) for a in compute_steps(i, p, step_fraction=s)]}
        for i, p, s in STEP_CASES
    ]
    (HERE / "geometry.json").write_text(json.dumps(geometry, indent=1) + "\n")

    arrays: dict[str, np.ndarray] = {}
    for patch in GAUSSIAN_FULL:
        arrays["full_" + "x".join(map(str, patch))] = gaussian_importance(patch)
    for patch in GAUSSIAN_SUMMARY:
        g = gaussian_importance(patch)
        name = "x".join(map(str, patch))
        c = tuple(s // 2 for s in patch)
        arrays[f"line0_{name}"] = g[:, c[1], c[2]].copy()
        arrays[f"line1_{name}"] = g[c[0], :, c[2]].copy()
        arrays[f"line2_{name}"] = g[c[0], c[1], :].copy()
        arrays[f"stats_{name}"] = np.array(
            [g.max(), g.min(), g.astype(np.float64).sum()], dtype=np.float64)
    for patch in FP16_GAUSSIAN:
        arrays["fp16_" + "x".join(map(str, patch))] = nnunet_fp16_gaussian(patch)
    np.savez_compressed(HERE / "gaussian.npz", **arrays)

    rng = np.random.default_rng(7)
    cases = {
        "plain": _upstream_plain_keys(3, (2, 2, 2), (2, 2), 2, (4, 8, 16), 3),
        "residual": _upstream_residual_keys(1, (4, 8, 16), (1, 2, 2), 3),
    }
    wmap = {}
    layouts: dict[str, np.ndarray] = {}
    for name, shapes in cases.items():
        state = {k: _Tensor(rng.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}
        converted = convert_state_dict(state)
        entries = {}
        for key, tensor in state.items():
            mapped = map_key_and_layout(key, tensor.array)
            entries[key] = None if mapped is None else mapped[0]
            if mapped is not None and key.endswith(("transpconvs.0.weight", "stages.0.0.convs.0.conv.weight",
                                                    "blocks.0.skip.1.conv.weight", "seg_layers.0.weight")):
                layouts[f"{name}|{key}|source"] = tensor.array
                layouts[f"{name}|{key}|converted"] = np.ascontiguousarray(mapped[1])
        wmap[name] = {"entries": entries, "dropped": list(converted.dropped_keys),
                      "converted_keys": sorted(converted.weights),
                      "source_shapes": {k: list(v) for k, v in shapes.items()}}
    (HERE / "weights_map.json").write_text(json.dumps(wmap, indent=1, sort_keys=True) + "\n")
    np.savez_compressed(HERE / "weights_layout.npz", **layouts)

    recorded = np.load(reference / "tests" / "fixtures" / "darwin-arm64" / "upstream_runner.npz")
    subset = {k: recorded[k] for k in recorded.files if k.startswith(("head_", "rounding_"))}
    # the reference's own host conversion of the recorded logits, as a cross-check
    subset["reference_probabilities_class"] = inference.logits_to_probabilities(
        recorded["head_logits_class"], has_regions=False)
    np.savez_compressed(HERE / "upstream_runner_subset.npz", **subset)

    from nnunet_mlx.data.resampling import separate_z_axis
    from nnunet_mlx.kernels.metal_restore import _axis_metadata, device_class_restore_supported
    from nnunet_mlx.plans import ResamplingContract

    axes: dict[str, np.ndarray] = {}
    for source, target in RESTORE_AXES:
        names = ("lower", "upper", "lower_high", "lower_low", "upper_high", "upper_low")
        for name, array in zip(names, _axis_metadata(source, target), strict=True):
            axes[f"{source}_{target}_{name}"] = array
    np.savez_compressed(HERE / "restore_axes.npz", **axes)
    support = []
    for source, target, current, new, (fn, order, order_z, force, threshold), classes in RESTORE_SUPPORT:
        contract = ResamplingContract(fn, order, order_z, force, separate_z_anisotropy_threshold=threshold)
        decision = device_class_restore_supported(source, target, current, new, contract, classes=classes)
        support.append({"source": list(source), "target": list(target), "current": list(current),
                        "new": list(new), "contract": [fn, order, order_z, force, threshold],
                        "classes": classes, "supported": bool(decision)})
    separate = []
    for current, new, force, threshold in SEPARATE_Z:
        flag, axis = separate_z_axis(current, new, force=force, threshold=threshold)
        separate.append({"current": list(current), "new": list(new), "force": force, "threshold": threshold,
                         "separate": bool(flag), "axis": axis})
    (HERE / "restore_policy.json").write_text(
        json.dumps({"support": support, "separate_z": separate}, indent=1) + "\n")

    # upstream torch-grid label resampling and recorded preprocessing runs (labels only: the
    # image inputs of those recordings are not tracked by the reference)
    recorded = np.load(reference / "tests" / "fixtures" / "darwin-arm64" / "torch_resampling.npz")
    metadata = json.loads(str(recorded["metadata"].item()))
    cases = [c for c in metadata["cases"] if f"{c['name']}-input" in recorded.files]
    labels = {k: recorded[k] for c in cases for k in (f"{c['name']}-input", f"{c['name']}-expected")}
    for run in metadata["pipeline"]:
        labels[f"{run['name']}-labels"] = recorded[f"{run['name']}-labels"]
    labels["raw_nonzero"] = recorded["raw_nonzero"]
    labels["previous"] = recorded["previous"]
    pipeline = [{k: run[k] for k in ("name", "plans", "properties", "geometry")} for run in metadata["pipeline"]]
    labels["metadata"] = np.array(json.dumps({"cases": cases, "pipeline": pipeline,
                                              "torch": metadata["torch"], "numpy": metadata["numpy"]}))
    np.savez_compressed(HERE / "torch_resampling_labels.npz", **labels)

    # half-pixel nearest indices of the out-of-plane pass (order 0) of spline resampling
    from nnunet_mlx.data.resampling import nearest_axis_indices

    nearest = [{"old": o, "new": n, "indices": [int(i) for i in nearest_axis_indices(o, n)]}
               for o, n in NEAREST_AXIS_CASES]
    (HERE / "nearest_axis.json").write_text(json.dumps(nearest) + "\n")

    # the reference's plan-entry parser and new-shape rounding, on accepted and rejected inputs
    from nnunet_mlx.data.resampling import compute_new_shape
    from nnunet_mlx.errors import ContractError as ReferenceContractError
    from nnunet_mlx.plans import ResamplingContract as ReferenceResampling

    entries = []
    for function, kwargs, expected_is_seg in PLAN_ENTRY_CASES:
        record = {"function": function, "kwargs": kwargs, "expected_is_seg": expected_is_seg}
        try:
            parsed = ReferenceResampling.from_configuration({"f": function, "f_kwargs": kwargs}, field="f",
                                                           expected_is_seg=expected_is_seg)
            record["parsed"] = {"function_name": parsed.function_name, "order": parsed.order,
                                "order_z": parsed.order_z, "force_separate_z": parsed.force_separate_z,
                                "seg_tiebreak": parsed.seg_tiebreak, "mode": parsed.mode,
                                "aniso_axis_mode": parsed.aniso_axis_mode,
                                "separate_z_anisotropy_threshold": parsed.separate_z_anisotropy_threshold}
        except ReferenceContractError:
            record["parsed"] = None
        entries.append(record)
    shapes = [{"shape": list(a), "old": list(b), "new": list(c), "result": list(compute_new_shape(a, b, c))}
              for a, b, c in NEW_SHAPE_CASES]
    (HERE / "preprocess_policy.json").write_text(json.dumps({"entries": entries, "new_shape": shapes}, indent=1)
                                                 + "\n")

    _record_reference_preprocessing(reference, recorded_plans=metadata["pipeline"][6]["plans"])
    _record_reference_plans(metadata)


def _record_reference_plans(metadata: dict) -> None:
    """The reference's ``PlansContract.from_payload`` view of every plans payload the fixtures hold."""
    from nnunet_mlx.plans import PlansContract

    payloads = [(f"pipeline:{i}", run["plans"]) for i, run in enumerate(metadata["pipeline"])]
    with np.load(HERE / "preprocess_reference.npz") as saved:
        cases = json.loads(str(saved["metadata"].item()))["cases"]
    payloads += [(f"reference:{i}", case["plans"]) for i, case in enumerate(cases)]
    spline_variants = []
    for order, order_z, force in ((3, 0, None), (1, 0, False), (3, 1, True)):
        plans = json.loads(json.dumps(metadata["pipeline"][8]["plans"]))
        config = plans["configurations"]["selected"]
        for field in ("resampling_fn_data", "resampling_fn_seg", "resampling_fn_probabilities"):
            config[field] = "resample_data_or_seg_to_shape"
            config[f"{field}_kwargs"] = {"is_seg": field == "resampling_fn_seg", "order": order,
                                         "order_z": order_z, "force_separate_z": force}
        spline_variants.append(plans)
    payloads += [(f"spline:{i}", plans) for i, plans in enumerate(spline_variants)]

    def entry(contract):
        return {"function_name": contract.function_name, "order": contract.order, "order_z": contract.order_z,
                "force_separate_z": contract.force_separate_z, "mode": contract.mode,
                "aniso_axis_mode": contract.aniso_axis_mode,
                "separate_z_anisotropy_threshold": contract.separate_z_anisotropy_threshold}

    parsed = []
    for name, plans in payloads:
        contract = PlansContract.from_payload(plans, configuration="selected")
        config = contract.configuration
        parsed.append({"name": name, "transpose_forward": list(contract.transpose_forward),
                       "transpose_backward": list(contract.transpose_backward), "spacing": list(config.spacing),
                       "normalization_schemes": list(config.normalization_schemes),
                       "use_mask_for_norm": list(config.use_mask_for_norm),
                       "data": entry(config.data_resampling), "seg": entry(config.segmentation_resampling),
                       "probabilities": entry(config.probability_resampling)})
    (HERE / "plans_reference.json").write_text(json.dumps({"spline_variants": spline_variants, "parsed": parsed})
                                               + "\n")


def _load_reference_preprocessing(reference: Path):
    """The reference's ``data/preprocessing.py`` as a module.

    Its one Python-3.13-only construct (a default on the generic parameter of
    ``PreprocessedRawCase``) is dropped in memory so that the module runs on 3.12;
    nothing else changes and nothing is written.
    """
    import types

    path = reference / "src" / "nnunet_mlx" / "data" / "preprocessing.py"
    source = path.read_text().replace("class PreprocessedRawCase[T = FloatArray]:", "class PreprocessedRawCase[T]:")
    module = types.ModuleType("nnunet_mlx.data.preprocessing")
    module.__file__ = str(path)
    sys.modules["nnunet_mlx.data.preprocessing"] = module
    exec(compile(source, str(path), "exec"), module.__dict__)
    return module


def _record_reference_preprocessing(reference: Path, *, recorded_plans: dict) -> None:
    """``preprocess_raw_case`` outputs of the reference for grid-preserving plans (no resampler needed)."""
    from nnunet_mlx.plans import PlansContract

    module = _load_reference_preprocessing(reference)
    rng = np.random.default_rng(77)
    ct = {"mean": 60.5, "std": 41.25, "percentile_00_5": -150.0, "percentile_99_5": 230.0}
    arrays: dict[str, np.ndarray] = {}
    cases = []
    for name, dtype, schemes, use_mask, transpose, cascade in PREPROCESS_CASES:
        channels = len(schemes)
        shape = (channels, 9, 11, 10)
        values = np.zeros(shape, dtype=np.float64)
        values[:, 1:8, 2:10, 1:9] = rng.normal(40, 90, (channels, 7, 8, 8))
        values[:, 4, 5, 4] = 0  # an enclosed hole of the nonzero mask
        if "RGBTo01Normalization" in schemes:
            values = np.clip(np.abs(values), 0, 255)
        if np.dtype(dtype).kind in "iu":
            values = np.round(values)
        raw = values.astype(dtype)
        plans = json.loads(json.dumps(recorded_plans))
        plans["transpose_forward"] = list(transpose)
        plans["transpose_backward"] = [list(transpose).index(a) for a in range(3)]
        plans["foreground_intensity_properties_per_channel"] = {str(c): dict(ct) for c in range(channels)}
        config = plans["configurations"]["selected"]
        config.update({"spacing": [None, None, None], "normalization_schemes": list(schemes),
                       "use_mask_for_norm": list(use_mask)})
        previous = rng.integers(0, 3, (1, *shape[1:])).astype(np.int16) if cascade else None
        spacing = [0.7, 1.6, 5.0]
        out = module.preprocess_raw_case(raw, {"spacing": spacing},
                                         PlansContract.from_payload(plans, configuration="selected"),
                                         segmentation_previous_stage=previous)
        arrays[f"{name}-raw"] = raw
        arrays[f"{name}-data"] = np.asarray(out.data)
        if previous is not None:
            arrays[f"{name}-previous"] = previous
            arrays[f"{name}-labels"] = np.asarray(out.previous_stage)
        cases.append({"name": name, "plans": plans, "spacing": spacing,
                      "bbox": out.properties["bbox_used_for_cropping"],
                      "shape_before_cropping": list(out.properties["shape_before_cropping"])})
    arrays["metadata"] = np.array(json.dumps({"cases": cases}))
    np.savez_compressed(HERE / "preprocess_reference.npz", **arrays)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the nnunet-mlx checkout>")
    main(Path(sys.argv[1]))
