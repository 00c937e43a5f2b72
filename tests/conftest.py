"""Shared pytest setup: import paths, the ``gpu`` marker, fixtures."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "paged-decode-lab_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        with np.load(GOLDEN / f"{name}.npz") as data:
            return {key: data[key] for key in data.files}
    return load
