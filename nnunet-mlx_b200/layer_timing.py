"""Per-layer device timing of one network forward (CUDA events around every library call).

    python -m nnunet_mlx_b200.layer_timing --config 2 --precision fp32 --batch 8 --patch 128

Builds a benchmark configuration's network with seeded synthetic weights, runs
``--warmup`` untimed forwards on a random ``(batch, patch^3, channels)`` input,
then one forward with the library profiler on, and prints one line per device
call (operation, shape, milliseconds, useful TFLOP/s or GB/s).  The batch of 8
is one tile's 8 mirror views.  Also the small driver used for single-kernel
ncu captures (``--batch 1``).
"""

from __future__ import annotations

import argparse
import json

import torch

from nnunet_mlx_b200 import _native, kernels
from nnunet_mlx_b200.model.network import build_network
from nnunet_mlx_b200.synthetic import config_spec, seeded_weights


def time_forward(config: int, precision: str, batch: int, patch: int, warmup: int = 2,
                 device: str = "cuda:0") -> list[dict]:
    spec = config_spec(config)
    dev = torch.device(device)
    net = build_network(spec, precision=precision, device=dev).load_weights(seeded_weights(spec, 0))
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((batch, patch, patch, patch, spec.input_channels), device=dev, generator=gen)
    for _ in range(warmup):
        net(x)
    torch.cuda.synchronize()
    kernels.PROFILE.reset()
    kernels.PROFILE.enable(True)
    try:
        net(x)
        torch.cuda.synchronize()
    finally:
        kernels.PROFILE.enable(False)
    status, where = _native.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} at wait site {where}")
    return kernels.PROFILE.trace()


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", type=int, default=2)
    p.add_argument("--precision", choices=["fp32", "fp32-tf32x2", "tf32", "bf16"], default="fp32")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--patch", type=int, default=128)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--json", action="store_true", help="print the trace as JSON")
    args = p.parse_args(argv)
    trace = time_forward(args.config, args.precision, args.batch, args.patch, args.warmup)
    if args.json:
        print(json.dumps(trace))
        return
    total = 0.0
    for item in trace:
        ms = item["ms"]
        total += ms
        rate = (f"{item['flops'] / ms / 1e9:8.1f} TF/s" if item["flops"]
                else f"{item['bytes'] / ms / 1e6:8.1f} GB/s")
        print(f"{item['name']:24s} {item['detail'] or '':44s} {ms:9.3f} ms {rate}")
    print(f"{'total':24s} {'':44s} {total:9.3f} ms")


if __name__ == "__main__":
    main()
