"""Shared test setup: import paths, the `gpu` marker, common fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc

    orc.lib()
    return orc


@pytest.fixture(scope="session")
def ob():
    import orda_b200

    orda_b200.load_library()
    return orda_b200


def bf16_round(a):
    """Rounds an f32 array to the nearest bf16 value (ties to even), kept as f32."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).bfloat16().float().numpy()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
