"""Shared test setup: the `gpu` marker, import paths and fixture loaders.

Tests marked `gpu` need a CUDA device and the built library; everything
else runs on the CPU (`pytest -m "not gpu"`).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libexpertrelay_b200.so")


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    from expertrelay_b200 import _lib

    _lib.lib()
    return torch.device("cuda", 0)
