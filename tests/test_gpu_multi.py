"""Sharded sliding window on 2 GPUs (NCCL): every rank's z-slab equals the single-device result.

Runs only when at least two CUDA devices are visible; each rank is a spawned
process bound to its own GPU.  (fold, tile, view) units are split across the
ranks and reduce-scatters sum the accumulators, so the float32 sums differ
from the single-device order by rounding only.  The nnunet-fp16 mode shards
whole folds and must equal the single-device result bit for bit.
"""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_models(device):
    from nnunet_mlx_b200.model.network import build_network
    from nnunet_mlx_b200.model.topology import PlainConvUNetSpec
    from nnunet_mlx_b200.synthetic import seeded_weights

    k3 = (3, 3, 3)
    spec = PlainConvUNetSpec(input_channels=1, num_classes=3, features=(32, 64), kernel_sizes=(k3, k3),
                             strides=((1, 1, 1), (2, 2, 2)), encoder_convs=(2, 2), decoder_convs=(2,))
    return [build_network(spec, precision="fp32", device=device).load_weights(seeded_weights(spec, s))
            for s in (51, 52)]


def _worker(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist

    from nnunet_mlx_b200.distributed import predict_volume_sharded
    from nnunet_mlx_b200.prediction.sliding_window import predict_volume

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        models = _tiny_models(device)
        data = np.random.default_rng(61).standard_normal((1, 40, 36, 30)).astype(np.float32)
        volume = torch.from_numpy(data).to(device)
        z0, z1, logits, labels, invalid = predict_volume_sharded(
            models, volume, patch_size=(16, 16, 16), num_classes=3, mirroring_axes=(0, 1, 2))
        ref_logits, ref_labels = predict_volume(models, data, patch_size=(16, 16, 16), num_classes=3,
                                                mirroring_axes=(0, 1, 2), device=device)
        lo, hi = (z0, z1)
        spans = [None] * world
        dist.all_gather_object(spans, (lo, hi))
        covered = sorted(spans)
        assert covered[0][0] == 0 and covered[-1][1] == data.shape[1]
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
        if hi > lo:
            assert int(invalid.item()) == 0
            np.testing.assert_allclose(logits.cpu().numpy(), ref_logits[:, lo:hi].cpu().numpy(), rtol=1e-5,
                                       atol=1e-5)
            agree = (labels.cpu().numpy() == ref_labels[lo:hi].cpu().numpy()).mean()
            assert agree >= 0.9995, agree
        # nnunet-fp16: whole folds per rank, bitwise the single-device fold ensemble
        from nnunet_mlx_b200.distributed import predict_volume_fp16_sharded

        half, half_labels = predict_volume_fp16_sharded(models, volume, patch_size=(16, 16, 16), num_classes=3,
                                                        mirroring_axes=(0, 1, 2))
        ref_half, ref_half_labels = predict_volume(models, data, patch_size=(16, 16, 16), num_classes=3,
                                                   mirroring_axes=(0, 1, 2), device=device,
                                                   accumulation="nnunet-fp16")
        if rank == 0:
            assert torch.equal(half, ref_half) and torch.equal(half_labels, ref_half_labels)
        else:
            assert half is None and half_labels is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two CUDA devices")
def test_sharded_prediction_on_two_gpus_matches_single_device(cuda_device):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
