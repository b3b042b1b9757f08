"""Device timing of raw-case preprocessing on configuration 2's CT geometry.

    python -m nnunet_mlx_b200.preprocess_timing [--iters 20] [--cpu]

The raw case is the synthetic liver CT of the benchmark (int16 HU, 101 x 768 x 768, air -1000,
so the whole volume is nonzero) at spacing (5.0, 0.8, 0.8) mm, preprocessed for a plan with CT
normalisation (clip [-1000, 400], mean 100, std 50) and target spacing (5.0, 1.0, 1.0) mm on the
torch grid: the in-plane pass resamples 768 x 768 -> 614 x 614 (bilinear, the z axis kept; the
anisotropy policy names z as the separate axis, whose pass is the identity here).

One JSON line per kernel (mean of ``--iters`` launches after 3 warm-ups, CUDA events on the
launching stream; every input exceeds the 126 MB L2): algorithmic bytes, achieved GB/s and the
fraction of the measured HBM copy bandwidth.  A last line times the whole ``preprocess_raw_case``
call from a page-locked host int16 array (upload, bounds read-back, crop + normalise, resample,
error read-back), and the same call under nnU-Net's default spline plan (order 3, separate order-0 z);
the spline kernels' in-plane pass is timed on its own too.  ``--cpu`` adds the reference's host paths
for the same case (NumPy crop + CT normalisation in float32, then upstream's torch-CPU resampler with
all host threads; scipy's order-3 zoom per plane, one thread, on 8 planes scaled to the volume).
"""

from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path

import numpy as np
import torch

from nnunet_mlx_b200 import _native, kernels
from nnunet_mlx_b200.data.preprocessing import PreprocessingPlans, preprocess_raw_case
from nnunet_mlx_b200.synthetic import synthetic_ct_hu

SPACING = (5.0, 0.8, 0.8)
TARGET_SPACING = (5.0, 1.0, 1.0)
INTENSITY = {"0": {"mean": 100.0, "std": 50.0, "percentile_00_5": -1000.0, "percentile_99_5": 400.0}}


def plans(spline: bool = False) -> PreprocessingPlans:
    """Torch-grid plan, or nnU-Net's default spline plan (order 3, separate order-0 axis)."""
    if spline:
        function, kwargs = "resample_data_or_seg_to_shape", {"order": 3, "order_z": 0, "force_separate_z": None}
    else:
        function, kwargs = "resample_torch_fornnunet", {}
    payload = {"transpose_forward": [0, 1, 2], "foreground_intensity_properties_per_channel": INTENSITY,
               "configurations": {"3d_fullres": {
                   "spacing": list(TARGET_SPACING), "normalization_schemes": ["CTNormalization"],
                   "use_mask_for_norm": [False], "resampling_fn_data": function,
                   "resampling_fn_data_kwargs": {"is_seg": False, **kwargs}, "resampling_fn_seg": function,
                   "resampling_fn_seg_kwargs": {"is_seg": True, **kwargs}}}}
    return PreprocessingPlans.from_payload(payload, configuration="3d_fullres")


def hbm_peak() -> tuple[float, str]:
    path = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _timed(run, iters: int) -> float:
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        run()
    stop.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / iters


def _line(name: str, ms: float, nbytes: int, **extra) -> dict:
    peak, source = hbm_peak()
    gbs = nbytes / ms / 1e6
    return {"kernel": name, "ms": round(ms, 4), "bytes": int(nbytes), "gbs": round(gbs, 1),
            "hbm_frac": round(gbs / peak, 3), "peak": f"{peak} GB/s ({source})", **extra}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--cpu", action="store_true")
    args = p.parse_args(argv)
    device = torch.device("cuda:0")
    hu = synthetic_ct_hu()[None]  # (1, 101, 768, 768) int16
    raw = torch.from_numpy(hu).to(device)
    dims = list(hu.shape[1:])
    new_shape = (101, 614, 614)
    norm = [kernels.ChannelNormalization("CTNormalization", False, -1000.0, 400.0, 100.0, 50.0)]
    voxels = int(np.prod(dims))

    ms = _timed(lambda: kernels.nonzero_bounds(raw, (0, 1, 2)), args.iters)
    print(json.dumps(_line("nonzero_bounds", ms, voxels * 2 + 32, shape=dims, dtype="int16")), flush=True)

    out = {}

    def crop():
        out["x"], out["errors"] = kernels.crop_normalize(raw, (0, 1, 2), (0, 0, 0), dims, norm)
    ms = _timed(crop, args.iters)
    print(json.dumps(_line("crop_normalize (CT, fused)", ms, voxels * (2 + 4), shape=dims)), flush=True)

    x = out["x"]
    in_plane = lambda: kernels.torch_resize(x, new_shape, "linear")  # noqa: E731
    ms = _timed(in_plane, args.iters)
    print(json.dumps(_line("torch_resize (linear, in-plane)", ms, voxels * 4 + int(np.prod(new_shape)) * 4,
                           source=dims, target=list(new_shape))), flush=True)

    spline = lambda: kernels.nearest_axis_resize(  # noqa: E731
        kernels.spline_resize(x, new_shape, axes=0b110, order=3, float64_out=True), new_shape)
    ms = _timed(spline, args.iters)
    print(json.dumps(_line("spline_resize (order 3, in-plane, z kept) + rounding pass", ms,
                           voxels * 4 + int(np.prod(new_shape)) * 4, source=dims, target=list(new_shape),
                           note="bytes: float32 in + out only; the padded float64 coefficients "
                                f"({int(np.prod([101, 792, 792])) * 8} B) are written, prefiltered and read "
                                "on top")), flush=True)

    host = torch.from_numpy(hu).pin_memory()
    the_plans = plans()
    case = lambda: preprocess_raw_case(host, {"spacing": list(SPACING)}, the_plans, device=device)  # noqa: E731
    result = case()
    assert tuple(result.data.shape) == (1, *new_shape)
    ms = _timed(case, max(3, args.iters // 4))
    status, where = _native.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} at wait site {where}")
    line = {"call": "preprocess_raw_case (host int16 -> device float32)", "ms": round(ms, 3),
            "h2d_bytes": int(hu.nbytes), "raw_voxels_per_s": round(voxels / ms * 1e3)}
    if args.cpu:
        line["cpu"] = cpu_reference(hu, new_shape)
    print(json.dumps(line), flush=True)

    spline_plans = plans(spline=True)
    case = lambda: preprocess_raw_case(host, {"spacing": list(SPACING)}, spline_plans, device=device)  # noqa: E731
    assert tuple(case().data.shape) == (1, *new_shape)
    ms = _timed(case, max(3, args.iters // 4))
    line = {"call": "preprocess_raw_case, default spline plan (order 3, separate z)", "ms": round(ms, 3),
            "raw_voxels_per_s": round(voxels / ms * 1e3)}
    if args.cpu:
        line["cpu"] = cpu_spline_reference(hu, new_shape)
    print(json.dumps(line), flush=True)


def cpu_reference(hu: np.ndarray, new_shape) -> dict:
    """The reference's host path: NumPy crop + CT normalisation, then torch-CPU bilinear planes."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    mask = np.any(hu != 0, axis=0)
    bounds = [np.flatnonzero(np.any(mask, axis=tuple(o for o in range(3) if o != a))) for a in range(3)]
    box = tuple(slice(int(b[0]), int(b[-1]) + 1) for b in bounds)
    x = np.ascontiguousarray(hu[(slice(None), *box)], dtype=np.float32)
    np.clip(x, -1000.0, 400.0, out=x)
    x -= 100.0
    x /= 50.0
    planes = torch.from_numpy(x[0])[:, None]  # (z, 1, y, x): the in-plane pass on every plane
    torch.nn.functional.interpolate(planes, size=tuple(new_shape[1:]), mode="bilinear", align_corners=False)
    seconds = time.perf_counter() - t0
    return {"s_per_volume": round(seconds, 3), "cores": threads,
            "kind": "reference host path (NumPy normalisation + torch-CPU resampler)"}


def cpu_spline_reference(hu: np.ndarray, new_shape, planes: int = 8) -> dict:
    """The reference's host spline path (scipy zoom order 3 per plane, float64), 8 planes scaled."""
    from scipy import ndimage

    x = ((np.clip(hu[0, :planes].astype(np.float32), -1000.0, 400.0) - 100.0) / 50.0).astype(np.float32)
    t0 = time.perf_counter()
    for k in range(planes):
        ndimage.zoom(x[k].astype(np.float64), np.divide(new_shape[1:], x.shape[1:]), order=3, mode="nearest",
                     grid_mode=True)
    seconds = (time.perf_counter() - t0) * hu.shape[1] / planes
    return {"s_per_volume": round(seconds, 3), "cores": 1, "sample": f"{planes} of {hu.shape[1]} planes, scaled",
            "kind": "reference host path (scipy zoom order 3 per plane)"}


if __name__ == "__main__":
    main()
