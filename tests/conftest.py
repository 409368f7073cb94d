"""Shared pytest setup: markers, import paths, golden-fixture access."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: runs CUDA kernels on a B200 (sm_100a) GPU")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


def golden_cases():
    """(name, kind, params, inputs) from tests/golden/make_golden.py, inputs regenerated from seeds."""
    import make_golden

    return list(make_golden.cases())


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected a B200 (sm_100), found sm_{major}{minor}"
    import kernelcode_generate_b200 as kg

    kg.load()  # fails loudly when the sm_100a library is not built
    return torch.device("cuda:0")
