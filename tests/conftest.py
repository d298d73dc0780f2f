from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """Vectors produced by the reference implementation (tests/golden/make_golden.py)."""
    with np.load(GOLDEN / "reference_vectors.npz") as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def golden_baseline():
    import json

    meta = json.loads((GOLDEN / "golden_meta.json").read_text())
    with np.load(GOLDEN / "baseline_vectors.npz") as f:
        return meta["baseline"], {k: f[k] for k in f.files}
