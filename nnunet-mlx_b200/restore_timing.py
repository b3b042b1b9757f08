"""Device timing of the class-label restoration kernel on a benchmark-sized volume.

    python -m nnunet_mlx_b200.restore_timing [--case all|identity|resample|transposed|half] [--iters 20] [--cpu]

Cases, on configuration 2's CT geometry (101 x 768 x 768 crop, 3 classes):

* ``identity``: float32 logits already on the crop grid -> labels uncropped into 110 x 800 x 800;
* ``resample``: float32 logits on a coarser in-plane grid (101 x 614 x 614) -> 101 x 768 x 768,
  uncropped into 110 x 800 x 800;
* ``transposed``: ``resample`` with the output axes permuted (2, 0, 1);
* ``half``: ``resample`` with float16 logits.

Each case prints one JSON line: the mean launch time (CUDA events on the
launching stream around ``--iters`` back-to-back launches after 3 warm-ups;
the logits, 460-720 MB, exceed the 126 MB L2, so no flush is needed), the
algorithmic bytes (logits read once plus labels written), the achieved GB/s
and its fraction of the measured HBM copy bandwidth.  ``--cpu`` adds the
reference's host path for the same case (scipy order-1 ``zoom`` per class in
float64, then the first argmax, one thread) timed on an 8-plane slab and
scaled to the volume.
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import numpy as np
import torch

from nnunet_mlx_b200 import _native, kernels

CROP = (101, 768, 768)
VOLUME = (110, 800, 800)
LO = (4, 16, 16)
COARSE = (101, 614, 614)
CASES = {
    "identity": dict(source=CROP, axes=(0, 1, 2), dtype=torch.float32),
    "resample": dict(source=COARSE, axes=(0, 1, 2), dtype=torch.float32),
    "transposed": dict(source=COARSE, axes=(2, 0, 1), dtype=torch.float32),
    "half": dict(source=COARSE, axes=(0, 1, 2), dtype=torch.float16),
}
CLASSES = 3


def hbm_peak() -> tuple[float, str]:
    path = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def time_case(name: str, iters: int, device: torch.device) -> dict:
    case = CASES[name]
    gen = torch.Generator(device=device).manual_seed(0)
    logits = torch.randn((CLASSES, *case["source"]), device=device, generator=gen).to(case["dtype"])
    run = lambda: kernels.restore_class_labels(logits, CROP, class_axis=0, volume=VOLUME, crop_lo=LO,  # noqa: E731
                                               axes=case["axes"])
    for _ in range(3):
        labels, invalid = run()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        labels, invalid = run()
    stop.record(stream)
    torch.cuda.synchronize()
    if int(invalid.item()) != 0:
        raise RuntimeError("restoration reported non-finite values")
    status, where = _native.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} at wait site {where}")
    ms = start.elapsed_time(stop) / iters
    nbytes = logits.numel() * logits.element_size() + labels.numel() * labels.element_size()
    peak, source = hbm_peak()
    gbs = nbytes / ms / 1e6
    return {"case": name, "source": list(case["source"]), "crop": list(CROP), "volume": list(VOLUME),
            "axes": list(case["axes"]), "dtype": str(case["dtype"]).replace("torch.", ""), "classes": CLASSES,
            "ms": round(ms, 4), "bytes": int(nbytes), "gbs": round(gbs, 1),
            "hbm_frac": round(gbs / peak, 3), "peak": f"{peak} GB/s ({source})",
            "target_voxels_per_s": round(np.prod(CROP) / ms * 1e3)}


def cpu_sample(name: str) -> dict:
    """The host path (scipy zoom order 1 per class, float64, first argmax) on 8 planes, scaled to the volume."""
    from scipy import ndimage

    case = CASES[name]
    planes = 8
    source = (planes, *case["source"][1:])
    target = (planes, *CROP[1:])
    dtype = np.float16 if case["dtype"] == torch.float16 else np.float32
    logits = np.random.default_rng(0).standard_normal((CLASSES, *source)).astype(dtype)
    t0 = time.perf_counter()
    if source == target:
        values = logits.astype(np.float32)
    else:
        inp = logits if dtype == np.float32 else logits.astype(np.float64)
        values = np.stack([ndimage.zoom(inp[c], np.divide(target, source), order=1, mode="nearest", grid_mode=True)
                           for c in range(CLASSES)]).astype(dtype)
    np.argmax(values, axis=0).astype(np.uint16)
    seconds = (time.perf_counter() - t0) * CROP[0] / planes
    return {"case": name, "cpu_s_per_volume": round(seconds, 3), "cores": 1,
            "sample": f"{planes} of {CROP[0]} planes, scaled", "kind": "reference host path (scipy zoom)"}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--case", choices=["all", *CASES], default="all")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--cpu", action="store_true")
    args = p.parse_args(argv)
    device = torch.device("cuda:0")
    names = list(CASES) if args.case == "all" else [args.case]
    for name in names:
        line = time_case(name, args.iters, device)
        if args.cpu:
            line["cpu"] = cpu_sample(name)
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
