"""Upstream nnU-Net v2 trained-folder conversion (reference storage/upstream.py) on the host."""

from __future__ import annotations

import json
import os
import time

import numpy as np
import pytest
import torch

from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
from nnunet_mlx_b200.storage import upstream
from nnunet_mlx_b200.storage.checkpoint import read_state, read_weights
from nnunet_mlx_b200.storage.weights import convert_state_dict, expected_shapes

K3 = (3, 3, 3)
SPEC = PlainConvUNetSpec(input_channels=2, num_classes=3, features=(4, 8, 16), kernel_sizes=(K3,) * 3,
                         strides=((1, 1, 1), (2, 2, 2), (2, 2, 2)), encoder_convs=(2, 2, 2), decoder_convs=(2, 2),
                         conv_bias=True, norm_affine=True)


def _upstream_state(spec, seed):
    """dynamic-network-architectures PlainConvUNet state-dict names and shapes (torch layout)."""
    rng = np.random.default_rng(seed)
    shapes = {}
    ch, k = spec.input_channels, 3
    feats = spec.features
    for s in range(len(feats)):
        for c in range(spec.encoder_convs[s]):
            ci = ch if c == 0 else feats[s]
            p = f"encoder.stages.{s}.0.convs.{c}"
            shapes[f"{p}.conv.weight"] = (feats[s], ci, k, k, k)
            shapes[f"{p}.conv.bias"] = (feats[s],)
            shapes[f"{p}.norm.weight"] = (feats[s],)
            shapes[f"{p}.norm.bias"] = (feats[s],)
            shapes[f"{p}.all_modules.0.weight"] = (feats[s], ci, k, k, k)
        ch = feats[s]
    n = len(feats)
    for d in range(n - 1):
        below, skip = feats[n - 1 - d], feats[n - 2 - d]
        shapes[f"decoder.transpconvs.{d}.weight"] = (below, skip, 2, 2, 2)
        shapes[f"decoder.transpconvs.{d}.bias"] = (skip,)
        for c in range(spec.decoder_convs[d]):
            ci = 2 * skip if c == 0 else skip
            p = f"decoder.stages.{d}.convs.{c}"
            shapes[f"{p}.conv.weight"] = (skip, ci, k, k, k)
            shapes[f"{p}.conv.bias"] = (skip,)
            shapes[f"{p}.norm.weight"] = (skip,)
            shapes[f"{p}.norm.bias"] = (skip,)
        shapes[f"decoder.seg_layers.{d}.weight"] = (spec.num_classes, skip, 1, 1, 1)
        shapes[f"decoder.seg_layers.{d}.bias"] = (spec.num_classes,)
    return {key: torch.from_numpy(rng.standard_normal(shape).astype(np.float32)) for key, shape in shapes.items()}


def _trained_folder(root, folds=(0, 1), trainer="nnUNetTrainer", mirroring=(0, 1, 2)):
    from nnunet_mlx_b200.synthetic import _plans_payload

    folder = root / "Dataset007_Test" / f"{trainer}__nnUNetPlans__3d_fullres"
    folder.mkdir(parents=True)
    (folder / "plans.json").write_text(json.dumps(_plans_payload(SPEC, (32, 32, 32), "3d_fullres")))
    dataset = {"channel_names": {"0": "CT", "1": "PET"}, "labels": {"background": 0, "a": 1, "b": 2},
               "numTraining": 3, "file_ending": ".nii.gz"}
    (folder / "dataset.json").write_text(json.dumps(dataset))
    states = {}
    for fold in folds:
        states[fold] = _upstream_state(SPEC, 10 + (fold if isinstance(fold, int) else 9))
        (folder / f"fold_{fold}").mkdir()
        torch.save({"network_weights": states[fold], "init_args": {"configuration": "3d_fullres", "fold": fold},
                    "trainer_name": trainer, "inference_allowed_mirroring_axes": mirroring,
                    "current_epoch": 1000,
                    "logging": {"ema_fg_dice": [np.float64(0.5), np.float32(0.7)], "epoch": np.int64(3)}},
                   folder / f"fold_{fold}" / "checkpoint_final.pth")
    return folder, states


def test_convert_trained_model_writes_a_loadable_folder(tmp_path):
    folder, states = _trained_folder(tmp_path)
    result = upstream.convert_trained_model(folder, tmp_path / "converted")
    assert result.folds == (0, 1) and result.configuration == "3d_fullres"
    out = result.folder
    assert (out / "plans.json").read_bytes() == (folder / "plans.json").read_bytes()
    manifest = upstream.read_conversion_manifest(out)
    assert [e["fold"] for e in manifest["folds"]] == [0, 1]
    for fold in (0, 1):
        directory = out / f"fold_{fold}" / "checkpoint_final"
        state = read_state(directory)
        assert state.identity.fold == fold and state.identity.trainer_name == "nnUNetTrainer"
        assert state.inference_allowed_mirroring_axes == (0, 1, 2)
        weights = read_weights(directory)
        assert set(weights) == set(expected_shapes(SPEC))
        expect = convert_state_dict(states[fold]).weights
        for key, value in weights.items():
            np.testing.assert_array_equal(value, expect[key])
        # a conv weight moved from torch (Co, Ci, kD, kH, kW) to (Co, kD, kH, kW, Ci)
        torch_w = states[fold]["encoder.stages.0.0.convs.0.conv.weight"].numpy()
        np.testing.assert_array_equal(weights["enc0.block0.conv.weight"], np.transpose(torch_w, (0, 2, 3, 4, 1)))


def test_no_mirroring_trainer_and_fold_selection(tmp_path):
    folder, _ = _trained_folder(tmp_path, folds=(0, 2, "all"), trainer="nnUNetTrainerNoMirroring", mirroring=None)
    assert upstream.detect_upstream_folds(folder) == (0, 2, "all")
    result = upstream.convert_trained_model(folder, tmp_path / "c", folds=["2", "all"])
    assert result.folds == (2, "all")
    assert read_state(result.folder / "fold_all" / "checkpoint_final").inference_allowed_mirroring_axes == ()


def test_rejections(tmp_path):
    folder, states = _trained_folder(tmp_path / "a", trainer="nnUNetTrainerBN")
    with pytest.raises(ContractError, match="not supported"):
        upstream.convert_trained_model(folder, tmp_path / "x")
    folder, states = _trained_folder(tmp_path / "b")
    bad = dict(states[0])
    bad.pop("decoder.seg_layers.1.bias")
    torch.save({"network_weights": bad, "init_args": {"configuration": "3d_fullres"}, "trainer_name": "nnUNetTrainer",
                "inference_allowed_mirroring_axes": (0, 1, 2)}, folder / "fold_0" / "checkpoint_final.pth")
    with pytest.raises(ContractError, match="do not match"):
        upstream.convert_trained_model(folder, tmp_path / "y")
    assert not (tmp_path / "y").exists()
    # arbitrary pickled objects are refused by the restricted unpickler
    torch.save({"network_weights": states[1], "init_args": {"configuration": "3d_fullres"},
                "trainer_name": "nnUNetTrainer", "inference_allowed_mirroring_axes": (0, 1, 2),
                "extra": ContractError("not allowed")}, folder / "fold_1" / "checkpoint_final.pth")
    with pytest.raises(ContractError, match="unreadable"):
        upstream.load_upstream_checkpoint(folder / "fold_1" / "checkpoint_final.pth")


def test_cached_conversion_reuses_and_refreshes(tmp_path):
    folder, states = _trained_folder(tmp_path / "results")
    cache = tmp_path / "cache"
    first = upstream.cached_conversion(folder, cache=cache)
    stamp = (first / "conversion.json").stat().st_mtime_ns
    again = upstream.cached_conversion(folder, folds=[1], cache=cache)
    assert again == first and (first / "conversion.json").stat().st_mtime_ns == stamp
    # a retrained fold (new size / mtime) invalidates the cache entry
    time.sleep(0.01)
    ckpt = folder / "fold_1" / "checkpoint_final.pth"
    os.utime(ckpt, ns=(time.time_ns(), time.time_ns() + 10**9))
    refreshed = upstream.cached_conversion(folder, cache=cache)
    assert refreshed == first and (first / "conversion.json").stat().st_mtime_ns != stamp
    with pytest.raises(ContractError, match="folds"):
        upstream.cached_conversion(folder, folds=[4], cache=cache)


def test_resolve_results_folder(tmp_path, monkeypatch):
    folder, _ = _trained_folder(tmp_path / "results")
    monkeypatch.setenv("nnUNet_results", str(tmp_path / "results"))
    assert upstream.resolve_results_folder("7", configuration="3d_fullres") == folder
    assert upstream.resolve_results_folder("Dataset007_Test", configuration="3d_fullres") == folder
    with pytest.raises(ContractError):
        upstream.resolve_results_folder("8", configuration="3d_fullres")


def test_cli_resolves_upstream_models_through_the_cache(tmp_path, monkeypatch):
    from nnunet_mlx_b200 import cli

    folder, _ = _trained_folder(tmp_path / "results")
    monkeypatch.setenv("nnUNet_results", str(tmp_path / "results"))
    monkeypatch.setenv("NNUNET_MLX_CACHE", str(tmp_path / "cache"))
    args = cli.build_parser().parse_args(["predict", "-i", "in", "-o", "out", "-d", "7", "-chk", "checkpoint_final"])
    model, name = cli.resolve_model(args, None)
    assert name == "checkpoint_final" and (model / "conversion.json").is_file()
    assert model.parent.parent == tmp_path / "cache" / "converted"
    args = cli.build_parser().parse_args(["predict", "-i", "in", "-o", "out", "-m", str(model)])
    assert cli.resolve_model(args, None) == (model, "checkpoint_final")
    args = cli.build_parser().parse_args(["predict", "-i", "in", "-o", "out"])
    with pytest.raises(ContractError, match="exactly one"):
        cli.resolve_model(args, None)


@pytest.mark.gpu
def test_converted_folder_predicts_like_the_directly_loaded_network(cuda_device, tmp_path):
    from nnunet_mlx_b200.model.folder import load_model_bundle
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    folder, states = _trained_folder(tmp_path / "results")
    converted = upstream.convert_trained_model(folder, tmp_path / "converted").folder
    bundle = load_model_bundle(converted, configuration="3d_fullres", device=cuda_device)
    assert bundle.folds == (0, 1) and bundle.mirroring_axes == (0, 1, 2)
    direct = [build_network(SPEC, precision="fp32", device=cuda_device).load_weights(
        convert_state_dict(states[f]).weights) for f in (0, 1)]
    data = np.random.default_rng(3).standard_normal((2, 20, 36, 33)).astype(np.float32)
    kw = dict(patch_size=(16, 32, 32), num_classes=3, mirroring_axes=(0, 1, 2))
    got, got_labels = predict_volume(list(bundle.models), data, **kw)
    ref, ref_labels = predict_volume(direct, data, **kw)
    assert torch.equal(got, ref) and torch.equal(got_labels, ref_labels)
