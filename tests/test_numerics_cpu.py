"""Numerics of the default tensor-core mode, checked on the CPU.

The default ``fp32`` precision computes every tensor-core convolution from
fp16 operand pairs (``hi + lo``, three products, per-column power-of-two
weight scales).  Emulating exactly those products with float32 convolutions on
the benchmark network must stay inside the parity tolerance (logits within
rel/abs 1e-3 of float32, argmax >= 99.95%) with a wide margin, while a single
fp16 product per element must not -- the reason the pair exists.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from oracle import network as onet


def _case():
    from nnunet_mlx_b200.synthetic import config_spec, seeded_weights, synthetic_ct

    spec = config_spec(1)
    weights = seeded_weights(spec, 0)
    x = np.moveaxis(synthetic_ct((48, 96, 96), seed=1)[:, :, :48, :48], 0, -1)[None].copy()
    return spec, weights, x


def _forward_with(monkeypatch, spec, weights, x, conv3d, conv_transpose3d):
    with monkeypatch.context() as m:
        m.setattr(F, "conv3d", conv3d)
        m.setattr(F, "conv_transpose3d", conv_transpose3d)
        return onet.forward(x, weights, spec)


def test_fp16_pair_products_meet_the_logit_bound(monkeypatch):
    torch.set_num_threads(min(8, torch.get_num_threads()))
    spec, weights, x = _case()
    ref = onet.forward(x, weights, spec)
    got = _forward_with(monkeypatch, spec, weights, x, onet.fp16_pair_products(F.conv3d),
                        onet.fp16_pair_products(F.conv_transpose3d, transposed=True))
    err = np.abs(got - ref)
    assert err.max() <= 2.5e-4, err.max()          # 4x inside the 1e-3 bound
    assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.9995


def test_single_fp16_product_misses_the_bound(monkeypatch):
    spec, weights, x = _case()
    ref = onet.forward(x, weights, spec)

    def single(op):
        def conv(a, w, b=None, **kwargs):
            return op(a.half().float(), w.half().float(), b, **kwargs)
        return conv

    got = _forward_with(monkeypatch, spec, weights, x, single(F.conv3d), single(F.conv_transpose3d))
    assert np.abs(got - ref).max() > 1e-2


def test_fp16_pair_split_reproduces_values():
    t = torch.from_numpy(np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100)
    hi, lo = onet.fp16_pair(t)
    recon = hi.double() + lo.double()
    assert ((recon - t.double()).abs() <= 2.0 ** -21 * t.double().abs() + 2.0 ** -25).all()
