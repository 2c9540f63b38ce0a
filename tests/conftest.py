"""Shared pytest setup.

* ``gpu`` marks tests that need a CUDA device (run on a B200 with -m gpu);
  everything else runs on the CPU.
* ``router-ia_b200`` (the package root) and the repository root (for
  ``oracle``) go on ``sys.path``.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
SRC = REPO / "router-ia_b200"
for p in (str(SRC), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "reference_steps.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    data = np.load(GOLDEN)
    out = {k: data[k] for k in data.files}
    out["meta"] = json.loads(str(out["meta"]))
    return out


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)
