import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_meta():
    import json
    return json.loads((GOLDEN / "golden_meta.json").read_text())


@pytest.fixture(scope="session")
def golden_ago():
    """AGO fixtures from the reference's tests/reference_ago.py, with their metadata."""
    import json
    with np.load(GOLDEN / "golden_ago.npz") as z:
        data = {k: z[k] for k in z.files}
    data["_meta"] = json.loads((GOLDEN / "golden_ago_meta.json").read_text())
    return data


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
