"""Device timing of the HBM-bound kernels of the inference path at benchmark-configuration-2 sizes.

    python -m nnunet_mlx_b200.window_timing [--warmup 2] [--repeat 5] [--json]

Each case launches one kernel of the path on the sizes one step of the
benchmark (101 x 768 x 768 CT, 128^3 tiles of 8 mirrored views, 3 classes)
gives it, times ``--repeat`` launches with CUDA events after ``--warmup``
untimed ones, and reports the mean launch time with the achieved rate of its
algorithmic bytes (what the kernel must read and write once):

* ``gather_tiles_kernel``         8 mirrored views of a 128^3 tile from the volume;
* ``conv3d_first_kernel``         the 1 -> 32 first convolution of the 8 views;
* ``norm_finalize_kernel``        instance-norm statistics of that layer's per-tile partials;
* ``prepare_operand_kernel``      the fp16-pair operand of a 64^3 x 64 activation of 8 views;
* ``residual_join_kernel``        a residual block's join at 64^3 x 64, 8 views;
* ``conv_transpose_operand``      the decoder's last up-convolution 64^3 x 64 -> 128^3 x 32 of 8 views,
                                  written as the next convolution's fp16-pair operand;
* ``accumulate_tile_rows_kernel`` segmentation head + flip-back + Gaussian accumulation of one tile;
* ``normalize_labels_kernel``     normalise + labels + logits over the whole volume.

With ``--warmup 0 --repeat 1`` every kernel runs exactly once, which makes it
the driver of single-launch ncu captures; ``--only NAME`` runs one case.  Inputs are larger than L2 except the
partials of the finalize (a latency-bound reduction).  At most ~4 GB is held
on the device at a time.
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from nnunet_mlx_b200 import _native, kernels
from nnunet_mlx_b200.kernels import Lazy
from nnunet_mlx_b200.model.network import build_network
from nnunet_mlx_b200.prediction.sliding_window import VolumeAccumulator, mirror_masks, pad_minimum, tile_offsets
from nnunet_mlx_b200.synthetic import config_spec, seeded_weights

ROOT = Path(__file__).resolve().parent.parent


def _peak_gbs() -> float | None:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"])
    return None


def _time(launch, warmup: int, repeat: int) -> float:
    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeat):
        launch()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / repeat


def run(warmup: int = 2, repeat: int = 5, device: str = "cuda:0", only: str | None = None) -> list[dict]:
    dev = torch.device(device)
    torch.cuda.set_device(dev)
    spec = config_spec(2)
    net = build_network(spec, precision="fp32", device=dev).load_weights(seeded_weights(spec, 0))
    gen = torch.Generator(device=dev).manual_seed(0)
    patch = (128, 128, 128)
    masks = mirror_masks((0, 1, 2))
    views = len(masks)
    shape = (101, 768, 768)
    pads, crop = pad_minimum(shape, patch)
    pad_lo = tuple(a for a, _ in pads)
    spatial = tuple(s + a + b for s, (a, b) in zip(shape, pads))
    vox_tile = math.prod(patch)
    results = []

    def wanted(name):
        return only is None or only == name

    def record(name, detail, ms, nbytes):
        results.append({"kernel": name, "detail": detail, "ms": ms, "algorithmic_bytes": nbytes,
                        "gbs": nbytes / (ms / 1e3) / 1e9})

    # 1. gather of 8 views of the middle tile (reads 8 MB of volume per view, writes the batch)
    volume = torch.randn((1, *shape), device=dev, generator=gen)
    offset = tile_offsets(spatial, patch, 0.5)[60]
    batch = torch.empty((views, *patch, 1), device=dev)
    nonfinite = torch.zeros((1,), dtype=torch.int32, device=dev)
    items = [(offset, m) for m in masks]
    kernels.gather_tiles(volume, pad_lo, items, patch, out=batch, nonfinite=nonfinite)
    if wanted("gather_tiles_kernel"):
        ms = _time(lambda: kernels.gather_tiles(volume, pad_lo, items, patch, out=batch, nonfinite=nonfinite),
                   warmup, repeat)
        record("gather_tiles_kernel", "8 views of a 128^3 tile, 1 channel", ms, 2 * 4 * views * vox_tile)

    # 2. first convolution 1 -> 32 of the 8 views (+ its per-tile partials) and 3. their finalize
    layer = net.layers["enc0.block0"]
    holder = {}

    def first():
        holder["out"], holder["partials"] = kernels.conv3d(
            [Lazy(batch)], layer.weight, kernel=layer.kernel, stride=layer.stride, pad=layer.pad, cout=layer.cout,
            packed=layer.packed, precision=_native.PREC_FP32, slope=spec.leaky_slope)

    if wanted("conv3d_first_kernel") or wanted("norm_finalize_kernel"):
        ms = _time(first, warmup if wanted("conv3d_first_kernel") else 0, repeat if wanted("conv3d_first_kernel") else 1)
        if wanted("conv3d_first_kernel"):
            record("conv3d_first_kernel", "8 x 128^3, 1 -> 32, 3x3x3", ms, 4 * views * vox_tile * (1 + 32))
    if wanted("norm_finalize_kernel"):
        partials = holder["partials"]
        ms = _time(lambda: kernels.instance_norm_finalize(partials, layer.gamma, layer.beta, spec.norm_eps), warmup,
                   repeat)
        record("norm_finalize_kernel", f"partials {tuple(partials.shape)}", ms, 4 * partials.numel())
        del partials
    del holder, batch
    torch.cuda.empty_cache()

    # 4. operand preparation and 5. residual join of a 64^3 x 64 activation of 8 views
    raw = torch.randn((views, 64, 64, 64, 64), device=dev, generator=gen)
    scale = torch.rand((views, 64), device=dev, generator=gen) + 0.5
    shift = torch.randn((views, 64), device=dev, generator=gen)

    def prepare():
        kernels.prepare_operand(Lazy(raw, scale, shift, leaky=True), _native.PREC_FP32, spec.leaky_slope)

    if wanted("prepare_operand_kernel"):
        ms = _time(prepare, warmup, repeat)
        record("prepare_operand_kernel", "8 x 64^3 x 64, fp16 pairs", ms, 8 * raw.numel())
    if wanted("residual_join_kernel"):
        skip = torch.randn_like(raw)
        ms = _time(lambda: kernels.residual_join(Lazy(raw, scale, shift, leaky=False), Lazy(skip), spec.leaky_slope),
                   warmup, repeat)
        record("residual_join_kernel", "8 x 64^3 x 64", ms, 12 * raw.numel())
        del skip
    if wanted("conv_transpose_operand"):
        weight, bias, kernel, packed = net.up[len(spec.features) - 2]  # the last up-convolution: 64 -> 32
        lazy_in = Lazy(raw, scale, shift, leaky=True)
        kernels.prepare_operand(lazy_in, _native.PREC_FP32, spec.leaky_slope)  # prepared once, as in the network
        ms = _time(lambda: kernels.conv_transpose3d_operand(lazy_in, weight, bias, kernel, spec.leaky_slope,
                                                            packed=packed, precision=_native.PREC_FP32),
                   warmup, repeat)
        out_elems = views * 128 ** 3 * int(weight.shape[0])
        record("conv_transpose_operand", "8 x 64^3 x 64 -> 128^3 x 32, fp16-pair operand output", ms,
               4 * raw.numel() + 4 * out_elems)
        del lazy_in
    del raw, scale, shift
    torch.cuda.empty_cache()

    # 6. fused head + flip-back + Gaussian accumulation of one tile into the configuration-2 accumulator
    features = torch.randn((views, *patch, 32), device=dev, generator=gen)
    fscale = torch.rand((views, 32), device=dev, generator=gen) + 0.5
    fshift = torch.randn((views, 32), device=dev, generator=gen)
    lazy = Lazy(features, fscale, fshift, leaky=True)
    acc = VolumeAccumulator(spatial, spec.num_classes, patch, dev)
    if wanted("accumulate_tile_rows_kernel"):
        ms = _time(lambda: kernels.accumulate_tile(lazy, masks, net.seg_weight, net.seg_bias, acc.gaussian, acc.acc,
                                                   acc.normalizer, offset, add_normalizer=True,
                                                   slope=spec.leaky_slope), warmup, repeat)
        record("accumulate_tile_rows_kernel", "8 views x 128^3 x 32 features -> 3 classes", ms,
               4 * features.numel() + vox_tile * 2 * 4 * (spec.num_classes + 1) + 4 * vox_tile)
    del features, lazy
    torch.cuda.empty_cache()

    # 7. normalise + labels + logits over the cropped volume
    acc.acc.uniform_(-1, 1, generator=gen)
    acc.normalizer.uniform_(0.5, 1.5, generator=gen)
    lo = [c.start for c in crop]
    dims = [c.stop - c.start for c in crop]
    if wanted("normalize_labels_kernel"):
        ms = _time(lambda: kernels.normalize_labels(acc.acc, acc.normalizer, lo, dims, fold_divisor=1.0,
                                                    label_dtype=torch.uint8), warmup, repeat)
        vox = math.prod(dims)
        record("normalize_labels_kernel", "101 x 768 x 768, 3 classes -> float32 logits + uint8 labels", ms,
               vox * (4 * (spec.num_classes + 1) + 4 * spec.num_classes + 1))
    status, where = _native.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} at wait site {where}")
    return results


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--repeat", type=int, default=5)
    p.add_argument("--json", action="store_true")
    p.add_argument("--only", default=None, help="run one case (a kernel name above)")
    args = p.parse_args(argv)
    rows = run(args.warmup, max(1, args.repeat), only=args.only)
    peak = _peak_gbs()
    for row in rows:
        row["frac_of_measured_hbm"] = row["gbs"] / peak if peak else None
    if args.json:
        print(json.dumps(rows))
        return
    for row in rows:
        frac = f"{row['frac_of_measured_hbm']:.2f}" if row["frac_of_measured_hbm"] is not None else "-"
        print(f"{row['kernel']:30s} {row['ms']:8.3f} ms {row['gbs']:8.1f} GB/s  {frac} of HBM  {row['detail']}")


if __name__ == "__main__":
    main()
