"""Host logic of the fp16-pair operands (no GPU): operand-only activations and the volume range guard."""

from __future__ import annotations

import pytest
import torch

from nnunet_mlx_b200 import _native, kernels
from nnunet_mlx_b200.errors import ContractError
from nnunet_mlx_b200.kernels import Lazy


def test_operand_only_activation_refuses_float32_use():
    up = kernels.OperandOnly(torch.zeros((2, 4, 6, 8, 32)))
    assert up.channels == 32 and up.spatial == (4, 6, 8)
    assert _native.PREC_FP32 in up.prepared
    with pytest.raises(ContractError):
        up.segment()


@pytest.mark.parametrize("up_shape,skip_shape", [((8, 8, 8), (7, 8, 6)), ((6, 8, 8), (8, 8, 9))])
def test_match_spatial_keeps_operand_form(up_shape, skip_shape):
    from nnunet_mlx_b200.model.network import _match_spatial

    up = kernels.OperandOnly(torch.arange(2 * 32 * int(torch.tensor(up_shape).prod())).float().reshape(2, *up_shape, 32))
    skip = Lazy(torch.zeros((2, *skip_shape, 32)))
    matched = _match_spatial(up, skip)
    assert isinstance(matched, kernels.OperandOnly)
    assert matched.spatial == skip_shape
    plain = _match_spatial(Lazy(up.raw), skip)
    assert not isinstance(plain, kernels.OperandOnly)
    torch.testing.assert_close(matched.raw, plain.raw)  # the same crop / zero pad of the buffer


class _FakeNet:
    def __init__(self, name, guarded):
        self.name, self.range_guarded = name, guarded

    def range_fallback(self):
        return _FakeNet(self.name + "-tf32x2", False)


@pytest.mark.parametrize("events,expect", [(0, ["a"]), (3, ["a", "a-tf32x2"])])
def test_range_guard_recomputes_with_split_tf32_twins(monkeypatch, events, expect):
    from nnunet_mlx_b200.prediction import sliding_window

    counter = {"reads": 0}

    def fake_events(reset=False):
        counter["reads"] += 1
        return events if counter["reads"] > 1 else 0  # reset read first, then the volume's count

    monkeypatch.setattr(kernels, "operand_range_events", fake_events)
    runs = []
    result = sliding_window.range_guarded([_FakeNet("a", True)], lambda ms: runs.append(ms[0].name) or ms[0].name)
    assert runs == expect and result == expect[-1]


def test_range_guard_skips_unguarded_precisions(monkeypatch):
    from nnunet_mlx_b200.prediction import sliding_window

    monkeypatch.setattr(kernels, "operand_range_events", lambda reset=False: pytest.fail("no guard expected"))
    assert sliding_window.range_guarded([_FakeNet("b", False)], lambda ms: "ran") == "ran"
