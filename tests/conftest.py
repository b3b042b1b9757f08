"""Test configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on any machine (oracle vs golden vectors, host logic,
C-ABI exports).  ``-m gpu`` needs a B200 and compares the CUDA path, called
through the C ABI, with the CPU oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA extension")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nnunet_mlx_b200 import build

    build.build_extension()
    major, minor = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"the CUDA path targets sm_100a; found sm_{major}{minor}")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, the device status word must be clear (no expired waits)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from nnunet_mlx_b200 import _native

    torch.cuda.synchronize()
    status, where = _native.device_status(reset=True)
    assert status == 0, f"device-side check failed: status {status} at wait site {where}"
