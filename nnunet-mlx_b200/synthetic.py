"""Seeded networks, synthetic volumes and model folders for the benchmark configurations.

The reference measures on released models and real CT/MRI/PET cases that are
not available here; these generators stand in with the same shapes, channel
counts, class counts and value distributions:

* ``config_spec(n)``    -- the network of benchmark configuration ``n`` (1..5);
* ``seeded_weights``    -- Kaiming-normal (fan-in, gain sqrt(2)) convolution and
                           transposed-convolution weights from a NumPy seed,
                           zero biases, norm gamma = 1 and beta = 0;
* ``synthetic_ct`` / ``synthetic_mri`` / ``synthetic_pet_ct`` -- preprocessed
  ``(C, z, y, x)`` float32 volumes;
* ``write_model_folder`` -- a converted model folder (``plans.json``,
  ``dataset.json``, ``fold_k/checkpoint_final``) in the reference's format.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from nnunet_mlx_b200.model.topology import NetworkSpec, PlainConvUNetSpec, ResidualEncoderUNetSpec
from nnunet_mlx_b200.storage.checkpoint import (
    CheckpointIdentity,
    InferenceCheckpointState,
    save_inference_checkpoint,
)
from nnunet_mlx_b200.storage.weights import expected_shapes

FEATURES = (32, 64, 128, 256, 320, 320)
PATCH = (128, 128, 128)


def plain_spec(input_channels: int, num_classes: int, *, features=FEATURES,
               patch_stages: int | None = None) -> PlainConvUNetSpec:
    stages = len(features) if patch_stages is None else patch_stages
    features = tuple(features[:stages])
    return PlainConvUNetSpec(
        input_channels=input_channels, num_classes=num_classes, features=features,
        kernel_sizes=((3, 3, 3),) * stages,
        strides=((1, 1, 1),) + ((2, 2, 2),) * (stages - 1),
        encoder_convs=(2,) * stages, decoder_convs=(2,) * (stages - 1), conv_bias=True)


def resenc_spec(input_channels: int, num_classes: int) -> ResidualEncoderUNetSpec:
    return ResidualEncoderUNetSpec(
        input_channels=input_channels, num_classes=num_classes, features=FEATURES,
        kernel_sizes=((3, 3, 3),) * 6, strides=((1, 1, 1),) + ((2, 2, 2),) * 5,
        encoder_blocks=(1, 3, 4, 6, 6, 6), decoder_convs=(1,) * 5, conv_bias=True)


CONFIGS = {
    1: {"spec": lambda: plain_spec(1, 3), "seeds": (0,), "mirror": ()},
    2: {"spec": lambda: plain_spec(1, 3), "seeds": (0,), "mirror": (0, 1, 2)},
    3: {"spec": lambda: plain_spec(4, 5), "seeds": (10, 11, 12, 13, 14), "mirror": (0, 1, 2)},
    4: {"spec": lambda: plain_spec(2, 2), "seeds": (20, 21, 22, 23, 24), "mirror": (0, 1, 2)},
    5: {"spec": lambda: resenc_spec(1, 3), "seeds": (30,), "mirror": (0, 1, 2)},
}


def config_spec(number: int) -> NetworkSpec:
    return CONFIGS[number]["spec"]()


def seeded_weights(spec: NetworkSpec, seed: int) -> dict[str, np.ndarray]:
    """Kaiming-normal weights in the converted layout, generated in parameter build order."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for key, shape in expected_shapes(spec).items():
        if key.endswith("norm.weight"):
            out[key] = np.ones(shape, np.float32)
        elif key.endswith("bias"):
            out[key] = np.zeros(shape, np.float32)
        else:
            # (C_out, *kernel, C_in): every output sums C_in * prod(kernel) products,
            # except a stride == kernel transposed conv where each output sees C_in.
            fan_in = shape[-1] if key.startswith("up") else int(np.prod(shape[1:]))
            std = np.sqrt(2.0 / fan_in)
            out[key] = (rng.standard_normal(shape) * std).astype(np.float32)
    return out


def _ellipsoids(rng, shape, count, radius_range):
    """Yield (slices, mask) of random axis-aligned ellipsoids inside ``shape``."""
    for _ in range(count):
        radii = [int(rng.integers(max(2, int(s * radius_range[0])), max(3, int(s * radius_range[1]))))
                 for s in shape]
        center = [int(rng.integers(r, max(r + 1, s - r))) for r, s in zip(radii, shape)]
        sl = tuple(slice(max(0, c - r), min(s, c + r + 1)) for c, r, s in zip(center, radii, shape))
        grids = np.ogrid[tuple(slice(s.start - c, s.stop - c) for s, c in zip(sl, center))]
        dist = sum((g.astype(np.float32) / max(r, 1)) ** 2 for g, r in zip(grids, radii))
        yield sl, dist <= 1.0


def synthetic_ct_hu(shape=(101, 768, 768), seed: int = 1) -> np.ndarray:
    """int16 HU: air -1000, 3-6 ellipsoid organs with mean U[20, 200] HU, noise sigma 15 HU."""
    rng = np.random.default_rng(seed)
    volume = np.full(shape, -1000.0, dtype=np.float32)
    for sl, mask in _ellipsoids(rng, shape, int(rng.integers(3, 7)), (0.08, 0.3)):
        volume[sl][mask] = rng.uniform(20, 200)
    volume += rng.standard_normal(shape, dtype=np.float32) * 15.0
    return np.clip(np.rint(volume), -32768, 32767).astype(np.int16)


def ct_normalize(hu: np.ndarray) -> np.ndarray:
    """Clip to [-1000, 400], then (x - 100) / 50 (the CT normalisation form of the configs)."""
    return ((np.clip(hu.astype(np.float32), -1000.0, 400.0) - 100.0) / 50.0).astype(np.float32)


def synthetic_ct(shape=(101, 768, 768), seed: int = 1) -> np.ndarray:
    return ct_normalize(synthetic_ct_hu(shape, seed))[None]


def _lowpass_noise(rng, shape) -> np.ndarray:
    from scipy.ndimage import gaussian_filter

    return gaussian_filter(rng.standard_normal(shape).astype(np.float32), sigma=4.0)


def _zscore_foreground(channel: np.ndarray) -> np.ndarray:
    threshold = np.percentile(channel, 5)
    mask = channel > threshold
    mean, std = channel[mask].mean(), channel[mask].std()
    return ((channel - mean) / max(std, 1e-8)).astype(np.float32)


def synthetic_mri(shape=(155, 240, 240), seed: int = 3) -> np.ndarray:
    """4-channel MRI: low-pass N(0,1) background + 2 ellipsoid lesions, z-scored per channel."""
    rng = np.random.default_rng(seed)
    lesions = list(_ellipsoids(rng, shape, 2, (0.05, 0.15)))
    channels = []
    for _ in range(4):
        channel = _lowpass_noise(rng, shape)
        for sl, mask in lesions:
            channel[sl][mask] += rng.uniform(0.5, 2.0)
        channels.append(_zscore_foreground(channel))
    return np.stack(channels)


def synthetic_pet_ct(shape=(284, 400, 400), seed: int = 4) -> np.ndarray:
    """2-channel PET/CT: CT as config 2, SUV = Exp(mean 0.5) + 5-20 Gaussian hotspots, / 10."""
    rng = np.random.default_rng(seed)
    ct = ct_normalize(synthetic_ct_hu(shape, seed + 100))
    suv = rng.exponential(0.5, size=shape).astype(np.float32)
    for _ in range(int(rng.integers(5, 21))):
        peak = rng.uniform(3, 20)
        sigma = rng.uniform(2, 6)
        center = [rng.uniform(0, s) for s in shape]
        r = int(3 * sigma) + 1
        sl = tuple(slice(max(0, int(c) - r), min(s, int(c) + r + 1)) for c, s in zip(center, shape))
        grids = np.ogrid[sl]
        dist2 = sum((g - c) ** 2 for g, c in zip(grids, center))
        suv[sl] += (peak * np.exp(-0.5 * dist2 / sigma**2)).astype(np.float32)
    return np.stack([ct, suv / 10.0]).astype(np.float32)


def config_volume(number: int) -> np.ndarray:
    if number == 1:
        return np.random.default_rng(0).standard_normal((1, 128, 128, 128), dtype=np.float32)
    if number in (2, 5):
        return synthetic_ct()
    if number == 3:
        return synthetic_mri()
    if number == 4:
        return synthetic_pet_ct()
    raise ValueError(f"unknown configuration {number}")


def _plans_payload(spec: NetworkSpec, patch_size, configuration: str) -> dict:
    residual = isinstance(spec, ResidualEncoderUNetSpec)
    arch = {
        "features_per_stage": list(spec.features), "kernel_sizes": [list(k) for k in spec.kernel_sizes],
        "strides": [list(s) for s in spec.strides], "n_stages": len(spec.features),
        "n_conv_per_stage_decoder": list(spec.decoder_convs), "conv_bias": spec.conv_bias,
        "conv_op": "torch.nn.modules.conv.Conv3d", "norm_op": "torch.nn.modules.instancenorm.InstanceNorm3d",
        "norm_op_kwargs": {"eps": spec.norm_eps, "affine": spec.norm_affine},
        "dropout_op": None, "dropout_op_kwargs": None,
        "nonlin": "torch.nn.LeakyReLU", "nonlin_kwargs": {"inplace": True, "negative_slope": spec.leaky_slope},
    }
    if residual:
        arch["n_blocks_per_stage"] = list(spec.encoder_blocks)
        name = "dynamic_network_architectures.architectures.unet.ResidualEncoderUNet"
    else:
        arch["n_conv_per_stage"] = list(spec.encoder_convs)
        name = "dynamic_network_architectures.architectures.unet.PlainConvUNet"
    return {
        "dataset_name": "Dataset999_Synthetic", "plans_name": "nnUNetPlans",
        "configurations": {configuration: {
            "data_identifier": "nnUNetPlans_3d_fullres", "preprocessor_name": "DefaultPreprocessor",
            "batch_size": 2, "batch_dice": False, "patch_size": list(patch_size),
            "spacing": [1.0, 1.0, 1.0], "normalization_schemes": ["ZScoreNormalization"] * spec.input_channels,
            "use_mask_for_norm": [False] * spec.input_channels,
            "architecture": {"network_class_name": name, "arch_kwargs": arch,
                             "_kw_requires_import": ["conv_op", "norm_op", "dropout_op", "nonlin"]},
        }},
    }


def write_model_folder(folder: str | Path, spec: NetworkSpec, seeds, *, patch_size=PATCH,
                       configuration: str = "3d_fullres", mirroring_axes=(0, 1, 2)) -> Path:
    """Write a converted model folder with one fold per seed (folds 0..n-1)."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    (folder / "plans.json").write_text(json.dumps(_plans_payload(spec, patch_size, configuration), indent=1))
    labels = {"background": 0, **{f"class{i}": i for i in range(1, spec.num_classes)}}
    dataset = {"channel_names": {str(i): f"ch{i}" for i in range(spec.input_channels)},
               "labels": labels, "numTraining": 0, "file_ending": ".nii.gz"}
    (folder / "dataset.json").write_text(json.dumps(dataset, indent=1))
    for fold, seed in enumerate(seeds):
        state = InferenceCheckpointState(
            identity=CheckpointIdentity("nnUNetTrainer", configuration, fold), current_epoch=None,
            spatial_dims=spec.spatial_dims, inference_allowed_mirroring_axes=tuple(mirroring_axes))
        save_inference_checkpoint(folder / f"fold_{fold}" / "checkpoint_final",
                                  weights=seeded_weights(spec, seed), state=state)
    return folder
