"""Shared test setup: import paths, the `gpu` marker, and lazily built native libraries."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "symwarp-fastdec_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def fdb():
    import fastdec_b200 as f
    if not f.LIB_PATH.exists():
        f.build()
    f.lib()
    return f


@pytest.fixture(scope="session")
def known():
    import json
    return json.loads((GOLDEN / "known_answers.json").read_text())


@pytest.fixture(scope="session")
def spiral_dm():
    import numpy as np
    sp = np.fromfile(GOLDEN / "spiral.f32", np.float32).reshape(-1, 2)
    return np.ascontiguousarray(sp.T)
