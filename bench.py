"""Benchmark: voxels/s of full-volume 8x-mirrored 3-D U-Net sliding-window inference on B200.

One step = one full pass of the inference hot path over the benchmark volume
(benchmark config 2: 1 x 101 x 768 x 768 synthetic CT, PlainConvUNet 32..320,
patch 128^3, step 0.5, 8 mirrored views, 1 fold; 121 tiles, 968 forwards):
mirrored tile gather -> U-Net forward of the 8 views as one batch -> fused seg
head + flip-back + Gaussian accumulation, for every tile; then normalise +
argmax into float32 logits and uint8 labels on the device.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

``value``: whole-job voxels/s with the preprocessed volume resident in HBM
(CUDA events on the compute stream, max over ranks).  ``e2e``: the same
metric through the public API with the volume in pinned host memory and the
float32 logits copied back each step, timed over as many steps as the device
figure.  ``--impl reference`` times the CPU restatement of the reference path
(oracle port; the reference itself needs MLX on Apple silicon) on the host
cores: each step is one full mirrored tile (every view's forward, the flips,
the Gaussian accumulation and the normalisation), extrapolated by the
volume's tile and fold counts.  Multi-GPU: launched with torchrun, one rank
per GPU; work units are sharded and the accumulators merged once with an
NCCL reduce-scatter, and ``check`` compares every rank's slab of a small crop
with a single-device prediction of the same crop.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "voxels/sec full-volume 3D U-Net inference (8x mirror TTA)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per launch of the dominant convolution launch, by precision, from the ncu
# captures summarised in profiles/: the z-streaming kernel (fp32) on the bench's own 8-view launch read
# 2274.9 MB (the raw input, 2147.5 MB, plus halo rows that missed L2) and wrote 2163.7 MB; split TF32 (halo
# kernel), captured on one view (views are independent samples of the batch, so an 8-view launch moves 8x
# that), read 537.2 MB (the hi/lo operand) and wrote 252.1 MB.
DOMINANT_TRAFFIC = {
    ("fp32", "8x128x128x128 32->32 k3x3x3 s1x1x1 conv3d_zstream_kernel"): 2274.894336e6 + 2163.651328e6,
    ("fp32-tf32x2", "8x128x128x128 32->32 k3x3x3 s1x1x1 conv3d_halo_kernel"): 8 * (537.210624e6 + 252.089088e6)}


# tensor products per useful product of each precision, relative to the dense bf16 rate
MODE_PRODUCTS = {"fp32": 3.0, "fp32-tf32x2": 8.0, "tf32": 2.0, "bf16": 1.0}
DTYPES = {"fp32": "fp32 (fp16-pair tensor-core products, fp32 accumulation)",
          "fp32-tf32x2": "fp32 (split-TF32 tensor cores)", "tf32": "tf32",
          "bf16": "bf16 inputs, fp32 accumulation"}
MODE_NOTES = {
    "fp32": "fp32 mode computes fp16 operand pairs: per 16-channel sub-step A_hi x W0, A_hi x W1 and A_lo x W0 "
            "(3 tensor products per useful product at the bf16/fp16 rate), so its arithmetic ceiling is peak/3",
    "fp32-tf32x2": "split TF32: 4 products at half the bf16 rate, ceiling peak/8",
    "tf32": "single-pass TF32: one product at half the bf16 rate, ceiling peak/2",
    "bf16": "bf16 operands, float32 accumulation: one product per useful product, ceiling = the dense bf16 peak",
}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--config", type=int, default=2, help="benchmark config number (2, 3, 4 or 5)")
    p.add_argument("--precision", choices=["fp32", "fp32-tf32x2", "tf32", "bf16"], default="fp32")
    p.add_argument("--e2e-steps", type=int, default=None, help="end-to-end steps (default: --steps)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-check", action="store_true", help="skip the sharded-vs-single-device slab check")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {**FALLBACK_PEAKS, "source": "fallback"}


def dominant_launch(trace):
    """The tensor-core convolution launch shape with the largest summed device time in ``trace``.

    Returns ``(detail, launches, mean_ms, flops_per_launch)`` or ``None``.
    """
    groups = {}
    for item in trace:
        if item["name"] != "conv3d_tc":
            continue
        g = groups.setdefault(item["detail"], [0, 0.0, item["flops"]])
        g[0] += 1
        g[1] += item["ms"]
    if not groups:
        return None
    detail, (count, total_ms, flops) = max(groups.items(), key=lambda kv: kv[1][1])
    return detail, count, total_ms / count, flops


def launch_table(trace, top: int = 10):
    """Per convolution launch shape (and kernel): launches, mean CUDA-event ms and useful TFLOP/s, largest total first."""
    groups = {}
    for item in trace:
        if item["name"] not in ("conv3d_tc", "conv_transpose3d_tc", "conv3d_simt"):
            continue
        g = groups.setdefault(item["detail"], [0, 0.0, item["flops"]])
        g[0] += 1
        g[1] += item["ms"]
    rows = sorted(groups.items(), key=lambda kv: -kv[1][1])[:top]
    return [{"launch": detail, "launches": n, "mean_ms": ms / n, "tflops": flops / (ms / n / 1e3) / 1e12}
            for detail, (n, ms, flops) in rows]


def forward_flops(spec, patch) -> float:
    """Algorithmic FLOPs (2 x MAC) of one network forward at ``patch`` (convs, transposed convs, seg head)."""
    from nnunet_mlx_b200.model.topology import ResidualEncoderUNetSpec

    flops = 0.0
    shape = list(patch)

    def conv(cin, cout, k, vox):
        return 2.0 * vox * cout * cin * math.prod(k)

    sizes = []
    if isinstance(spec, ResidualEncoderUNetSpec):
        stem = spec.effective_stem_channels
        vox = math.prod(shape)
        flops += conv(spec.input_channels, stem, spec.kernel_sizes[0], vox)
        cin = stem
        for s, f in enumerate(spec.features):
            shape = [a // b for a, b in zip(shape, spec.strides[s])]
            vox = math.prod(shape)
            sizes.append(list(shape))
            for b in range(spec.encoder_blocks[s]):
                bin_ = cin if b == 0 else f
                flops += conv(bin_, f, spec.kernel_sizes[s], vox) + conv(f, f, spec.kernel_sizes[s], vox)
                if b == 0 and bin_ != f:
                    flops += conv(bin_, f, (1, 1, 1), vox)
            cin = f
    else:
        cin = spec.input_channels
        for s, f in enumerate(spec.features):
            shape = [a // b for a, b in zip(shape, spec.strides[s])]
            vox = math.prod(shape)
            sizes.append(list(shape))
            for b in range(spec.encoder_convs[s]):
                flops += conv(cin if b == 0 else f, f, spec.kernel_sizes[s], vox)
            cin = f
    stages = len(spec.features)
    for d in range(stages - 1):
        src = stages - 1 - d
        below, skip = spec.features[src], spec.features[src - 1]
        vin = math.prod(sizes[src])
        vout = math.prod(sizes[src - 1])
        flops += 2.0 * vin * below * skip * math.prod(spec.strides[src])
        for b in range(spec.decoder_convs[d]):
            flops += conv(2 * skip if b == 0 else skip, skip, spec.kernel_sizes[src - 1], vout)
    flops += 2.0 * math.prod(sizes[0]) * spec.features[0] * spec.num_classes
    return flops


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_tile_seconds(spec, weights, axes, patch, threads: int) -> float:
    """Seconds for one full tile of the reference path on the host cores (the oracle port).

    One tile-sized volume through the oracle's sliding window: every mirrored
    view's forward, the flips back, the Gaussian accumulation and the
    normalisation (oracle/sliding_window.py restating the reference's
    ``predict_logits``).
    """
    import numpy as np
    import torch

    from oracle import network as onet
    from oracle import sliding_window as osw

    torch.set_num_threads(threads)
    tile = np.random.default_rng(0).standard_normal((spec.input_channels, *patch)).astype(np.float32)
    t0 = time.perf_counter()
    osw.predict_logits(lambda t: onet.forward(t, weights, spec), tile, patch_size=patch,
                       num_classes=spec.num_classes, mirroring_axes=axes)
    return time.perf_counter() - t0


def cpu_warm(spec, weights, threads: int) -> None:
    """One 64^3 forward of the oracle: warms the host thread pool and allocator."""
    import numpy as np
    import torch

    from oracle import network as onet

    torch.set_num_threads(threads)
    x = np.random.default_rng(1).standard_normal((1, 64, 64, 64, spec.input_channels)).astype(np.float32)
    onet.forward(x, weights, spec)


def cpu_rate(seconds: float, work: dict, folds: int) -> float:
    """Volume voxels/s implied by ``seconds`` per tile (tiles x folds tiles per volume)."""
    return work["voxels"] / (seconds * work["tiles"] * folds)


def cpu_sample_text(seconds: float, work: dict, folds: int, views: int, threads: int, patch) -> str:
    import torch

    return (f"one full {'x'.join(map(str, patch))} tile ({views} view forward(s) + flips + Gaussian "
            f"accumulation + normalisation, {seconds:.2f} s) on {threads} threads, extrapolated x{work['tiles']} "
            f"tiles x{folds} fold(s) (oracle/network.py + oracle/sliding_window.py, torch {torch.__version__} CPU)")


def cpu_baseline(spec, weights, axes, patch, work: dict, folds: int):
    """The CPU baseline of the repo arm: one timed full tile (as one step of ``--impl reference``)."""
    threads = host_threads()
    cpu_warm(spec, weights, threads)
    seconds = cpu_tile_seconds(spec, weights, axes, patch, threads)
    views = 2 ** len(axes)
    return {"value": cpu_rate(seconds, work, folds), "unit": "voxels/s", "cores": threads, "kind": "port",
            "sample": cpu_sample_text(seconds, work, folds, views, threads, patch)}


def bench_config(args, shape, patch, views: int, folds: int, work: dict, gflop: float, world: int) -> dict:
    """The ``config`` object both arms print (the same workload description)."""
    return {"workload": f"config{args.config}", "volume": list(shape), "patch": list(patch), "step_fraction": 0.5,
            "mirror_views": views, "folds": folds, "tiles": work["tiles"], "forwards": work["forwards"],
            "gflop_per_forward": gflop, "precision": args.precision,
            "l2": "inputs larger than L2 (each 128^3 layer reads and writes >= 268 MB per view)",
            "parallelism": f"tile-view units x folds sharded over {world} GPU(s)"}


def setup_distributed(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl != "reference":
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args, world, rank):
    """--impl reference: the CPU restatement of the reference path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from nnunet_mlx_b200.prediction.sliding_window import volume_work
    from nnunet_mlx_b200.synthetic import CONFIGS, config_spec, seeded_weights

    cfg = CONFIGS[args.config]
    spec = config_spec(args.config)
    weights = seeded_weights(spec, cfg["seeds"][0])
    patch = (128, 128, 128)
    axes = cfg["mirror"]
    views = 2 ** len(axes)
    folds = len(cfg["seeds"])
    shape = CONFIG_SHAPES[args.config]
    work = volume_work(shape, patch, 0.5, views, folds)
    threads = host_threads()
    for _ in range(args.warmup):
        cpu_warm(spec, weights, threads)
    times = [cpu_tile_seconds(spec, weights, axes, patch, threads) for _ in range(args.steps)]
    seconds = statistics.median(times)
    value = cpu_rate(seconds, work, folds)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic",
        "config": bench_config(args, shape, patch, views, folds, work, forward_flops(spec, patch) / 1e9, world),
        "step": "one full mirrored tile of the volume's workload; value = volume voxels / (median tile seconds x "
                "tiles x folds); warm-up steps run one 64^3 forward each to warm the thread pool",
        "seconds_per_volume_extrapolated": seconds * work["tiles"] * folds,
        "cpu_baseline": {"value": value, "unit": "voxels/s", "cores": threads, "kind": "port",
                         "sample": cpu_sample_text(seconds, work, folds, views, threads, patch)},
        "e2e": {"value": value, "unit": "voxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


CONFIG_SHAPES = {1: (128, 128, 128), 2: (101, 768, 768), 3: (155, 240, 240), 4: (284, 400, 400), 5: (101, 768, 768)}


def check_crop(host):
    """A small crop of the benchmark volume (<= 192 per axis, centred in y and x) for the slab check."""
    _, z, y, x = host.shape
    cz, cy, cx = min(z, 192), min(y, 192), min(x, 192)
    y0, x0 = (y - cy) // 2, (x - cx) // 2
    return host[:, :cz, y0:y0 + cy, x0:x0 + cx].copy()


def sharded_check(models, spec, host, axes, patch, device, world):
    """Every rank's slab of a sharded prediction of a crop against a single-device prediction of it."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from nnunet_mlx_b200.distributed import predict_volume_sharded
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    crop = check_crop(host)
    z0, z1, logits, labels, invalid = predict_volume_sharded(
        models, torch.from_numpy(crop).to(device), patch_size=patch, num_classes=spec.num_classes,
        mirroring_axes=axes)
    ref_logits, ref_labels = predict_volume(models, crop, patch_size=patch, num_classes=spec.num_classes,
                                            mirroring_axes=axes, device=device)
    err, disagree, bad, voxels = 0.0, 0, 0, 0
    if logits is not None:
        got = logits.cpu().numpy()
        ref = ref_logits[:, z0:z1].cpu().numpy()
        err = float(np.abs(got - ref).max())
        bad = int((~np.isclose(got, ref, rtol=1e-4, atol=1e-4)).sum()) + int(invalid.item())
        disagree = int((labels.cpu().numpy() != ref_labels[z0:z1].cpu().numpy()).sum())
        voxels = int(labels.numel())
    spans = torch.tensor([z0, z1], dtype=torch.int64, device=device)
    stats = torch.tensor([err], dtype=torch.float64, device=device)
    counts = torch.tensor([disagree, bad, voxels], dtype=torch.int64, device=device)
    covered = True
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        gathered = [torch.zeros_like(spans) for _ in range(world)]
        dist.all_gather(gathered, spans)
        pieces = sorted(tuple(int(v) for v in g.tolist()) for g in gathered)
        covered = pieces[0][0] == 0 and pieces[-1][1] == crop.shape[1] and all(
            a[1] == b[0] for a, b in zip(pieces, pieces[1:]))
    disagree, bad, voxels = (int(v) for v in counts.tolist())
    agreement = 1.0 - disagree / max(voxels, 1)
    return {"crop": list(crop.shape[1:]), "ranks": world, "max_abs_err": float(stats.item()),
            "values_outside_1e-4": bad, "argmax_agreement": agreement, "slabs_cover_crop": covered,
            "voxels_checked": voxels,
            "passed": bool(covered and bad == 0 and agreement >= 0.9995 and voxels == crop[0].size)}


def main():
    args = parse_args()
    world, rank, local = setup_distributed(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    from nnunet_mlx_b200 import _native, build, kernels
    from nnunet_mlx_b200.distributed import predict_volume_sharded
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.prediction.inference import ArrayPredictor
    from nnunet_mlx_b200.prediction.sliding_window import volume_work
    from nnunet_mlx_b200.synthetic import CONFIGS, config_spec, config_volume, seeded_weights

    build.build_extension()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = CONFIGS[args.config]
    spec = config_spec(args.config)
    patch = (128, 128, 128)
    weights = [seeded_weights(spec, seed) for seed in cfg["seeds"]]
    models = [build_network(spec, precision=args.precision, device=device).load_weights(w) for w in weights]
    host = config_volume(args.config)
    shape = host.shape[1:]
    axes = cfg["mirror"]
    views = 2 ** len(axes)
    work = volume_work(shape, patch, 0.5, views, len(models))
    volume = torch.from_numpy(host).to(device)

    def step():
        return predict_volume_sharded(models, volume, patch_size=patch, num_classes=spec.num_classes,
                                      mirroring_axes=axes, step_fraction=0.5)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    kernels.PROFILE.reset()
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kernels.PROFILE.enable(True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    kernels.PROFILE.enable(False)
    barrier()
    elapsed = start.elapsed_time(end) / 1e3
    if world > 1:
        t = torch.tensor([elapsed], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    status, where = _native.device_status(reset=True)
    if status != 0:
        raise SystemExit(f"device status {status} at wait site {where}")
    value = work["voxels"] * args.steps / elapsed
    prof = kernels.PROFILE.summary()
    dominant = dominant_launch(kernels.PROFILE.trace())

    # end to end through the public API: pinned host volume in, host logits out, as many steps as timed above
    e2e = None
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else args.steps
    if world == 1:
        predictor = ArrayPredictor(models, patch_size=patch, num_outputs=spec.num_classes, mirroring_axes=axes)
        pinned = torch.from_numpy(host).pin_memory()
        predictor.predict_logits_from_preprocessed_data(pinned)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            out = predictor.predict_logits_from_preprocessed_data(pinned)
        e2e_seconds = (time.perf_counter() - t0) / e2e_steps
        e2e = {"value": work["voxels"] / e2e_seconds, "unit": "voxels/s",
               "h2d_bytes_per_step": int(host.nbytes), "d2h_bytes_per_step": int(out.nbytes),
               "api": "ArrayPredictor.predict_logits_from_preprocessed_data", "steps": e2e_steps}
    else:
        pinned = torch.from_numpy(host).pin_memory()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            vol = pinned.to(device, non_blocking=True)
            z0, z1, logits, labels, invalid = predict_volume_sharded(
                models, vol, patch_size=patch, num_classes=spec.num_classes, mirroring_axes=axes)
            d2h = 0
            if logits is not None:
                d2h = kernels.to_host(logits).nbytes + kernels.to_host(labels).nbytes
        torch.cuda.synchronize()
        e2e_seconds = (time.perf_counter() - t0) / e2e_steps
        t = torch.tensor([e2e_seconds], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_seconds = float(t.item())
        total_d2h = torch.tensor([d2h], dtype=torch.int64, device=device)
        dist.all_reduce(total_d2h, op=dist.ReduceOp.SUM)
        e2e = {"value": work["voxels"] / e2e_seconds, "unit": "voxels/s",
               "h2d_bytes_per_step": int(host.nbytes) * world, "d2h_bytes_per_step": int(total_d2h.item()),
               "api": "distributed.predict_volume_sharded (pinned host volume per rank, slabs to host)",
               "steps": e2e_steps}

    check = None if args.no_check else sharded_check(models, spec, host, axes, patch, device, world)
    fwd = forward_flops(spec, patch)
    if rank == 0:
        pk = peaks()
        conv = prof.get("conv3d_tc", {})
        conv_all = conv.get("flops", 0.0) / conv["seconds"] / 1e12 if conv.get("seconds") else 0.0
        peak = pk["bf16_tflops_sustained"]
        ceiling = peak / MODE_PRODUCTS[args.precision]
        roofline = {"bound": "tensor", "kernel": None, "achieved": None, "peak": peak,
                    "unit": "TFLOP/s", "frac": None, "traffic": None}
        if dominant is not None:
            detail, count, mean_ms, flops = dominant
            achieved = flops / (mean_ms / 1e3) / 1e12
            roofline.update({
                "kernel": detail.rsplit(" ", 1)[-1], "launch": detail, "launches": count, "mean_ms": mean_ms,
                "achieved": achieved, "frac": achieved / peak,
                "traffic": DOMINANT_TRAFFIC.get((args.precision, detail)),
                "algorithmic_flops_per_launch": flops,
                "mode_ceiling": ceiling, "frac_of_mode_ceiling": achieved / ceiling,
                "all_conv_launches_tflops": conv_all})
        roofline.update({
            "peak_source": f"{pk['source']} dense bf16, sustained (kernel timed inside a long step)",
            "note": "achieved = algorithmic FLOPs (2 x MACs) of the dominant launch / its mean CUDA-event "
                    "duration over the timed region; " + MODE_NOTES[args.precision]})
        line = {
            "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": DTYPES[args.precision],
            "data": "synthetic",
            "config": bench_config(args, shape, patch, views, len(models), work, fwd / 1e9, world),
            "conv_tflops_effective": work["forwards"] * fwd * args.steps / elapsed / 1e12 / world,
            # the whole step against the tensor-core roof: algorithmic conv FLOPs per GPU / wall / sustained peak
            "step_roofline_frac": work["forwards"] * fwd * args.steps / elapsed / 1e12 / world / peak,
            "roofline": roofline,
            "kernels": prof,
            "conv_launches": launch_table(kernels.PROFILE.trace()),
            "clocks": clocks.summary(),
            "gpu_launches": kernels.PROFILE.launches,
            "e2e": e2e,
            "check": check,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(spec, weights[0], axes, patch, work, len(models))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
