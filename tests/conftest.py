"""Shared test setup.

Markers: ``gpu`` — needs a CUDA device (run on the B200 box with ``-m gpu``).
Everything unmarked runs on a CPU-only machine.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(REPO / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle():
    import slr_oracle

    slr_oracle.build()
    return slr_oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        # GPU tests never pass silently without a GPU: select them with -m gpu
        # on a CUDA machine, deselect them with -m "not gpu" elsewhere.
        pytest.fail("gpu-marked test run without a CUDA device")
    import s_salaad_b200

    s_salaad_b200.load()
    return torch.device("cuda:0")
