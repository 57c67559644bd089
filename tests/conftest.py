"""pytest configuration: the `gpu` marker and shared fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def golden():
    cache: dict[str, dict[str, np.ndarray]] = {}

    def load(name: str) -> dict[str, np.ndarray]:
        if name not in cache:
            with np.load(GOLDEN / f"{name}.npz") as data:
                cache[name] = {key: data[key] for key in data.files}
        return cache[name]

    return load


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is unavailable")
    return torch.device("cuda", 0)
