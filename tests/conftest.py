import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def load_golden(stem: str) -> dict:
    """Fixture file -> {case: {key: array}}."""
    data = np.load(GOLDEN / f"{stem}.npz")
    out: dict = {}
    for k in data.files:
        case, key = k.split(".", 1)
        out.setdefault(case, {})[key] = data[k]
    return out


@pytest.fixture(scope="session")
def golden():
    return load_golden
