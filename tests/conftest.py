"""Test configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the CPU suite (oracle against the golden vectors, the
C-ABI symbol table, host-side logic, gloo ranks); ``-m gpu`` runs the parity
tests on a B200 through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "tts-inference_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(ROOT / "tests" / "golden" / "quant_golden.npz"))


def require_b200():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.fail("these kernels need a compute-capability 10.x (B200) GPU")
