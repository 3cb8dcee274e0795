"""Test configuration: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need a B200 (sm_100) and the built libmgc_cuda.so; everything else runs on
the CPU (oracle vs golden fixtures, lowering, ABI symbol table, multi-process host logic).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "ml-graph-compiler_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and libmgc_cuda.so")
    config.addinivalue_line("markers", "slow: whole benchmark-size models")


def gpu_available() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available()) and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def golden_ops() -> dict:
    import numpy as np

    with np.load(ROOT / "tests" / "golden" / "ops.npz") as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def golden_models() -> dict:
    import numpy as np

    with np.load(ROOT / "tests" / "golden" / "models.npz") as f:
        return {k: f[k] for k in f.files}
