"""Shared test setup.

Markers: ``gpu`` — needs a CUDA device (run on the B200 box with ``-m gpu``).
Everything unmarked runs on a CPU-only machine.
"""
from __future__ import annotations

import json
import os
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


# ------------------------------------------------ achieved 16-bit error --

_PARITY_RECORDS: list[dict] = []


def record_parity(case: str, y, ref) -> float:
    """Record max|y - y_ref| / RMS(y_ref) of a 16-bit result under `case`."""
    y = y.float()
    ref = ref.float().to(y.device)
    rms = float(ref.pow(2).mean().sqrt())
    err = (y - ref).abs()
    worst = float(err.max()) if err.numel() else 0.0
    over = int((err > 2e-2 * rms).sum())
    ratio = worst / rms if rms else 0.0
    _PARITY_RECORDS.append({"case": case, "max_err_over_rms": ratio, "rms": rms, "outputs": int(err.numel()),
                            "over_2e-2_rms": over})
    return ratio


@pytest.fixture(scope="session")
def parity_log():
    """record_parity for the full-size cases (listed one by one at the end of
    the session; other 16-bit checks are summarised per test function)."""

    def log(name: str, y, ref) -> float:
        return record_parity("full size: " + name, y, ref)

    return log


def pytest_terminal_summary(terminalreporter):
    if not _PARITY_RECORDS:
        return
    tr = terminalreporter
    tr.section("16-bit parity: achieved max|err| / RMS(y_ref) (north_star bound 2e-2)")
    per_test: dict[str, dict] = {}
    for r in _PARITY_RECORDS:
        if r["case"].startswith("full size: "):
            tr.write_line(f"{r['case']:<60} {r['max_err_over_rms']:.3e}  outputs {r['outputs']:>10}  "
                          f"above 2e-2*RMS: {r['over_2e-2_rms']}")
            continue
        key = r["case"].split("[")[0]
        agg = per_test.setdefault(key, {"cases": 0, "worst": 0.0, "over": 0, "outputs": 0})
        agg["cases"] += 1
        agg["worst"] = max(agg["worst"], r["max_err_over_rms"])
        agg["over"] += r["over_2e-2_rms"]
        agg["outputs"] += r["outputs"]
    for key, agg in per_test.items():
        tr.write_line(f"{key:<60} worst {agg['worst']:.3e} over {agg['cases']} cases, {agg['outputs']} outputs; "
                      f"above 2e-2*RMS: {agg['over']}")
    out = os.environ.get("SLR_PARITY_LOG")
    if out:
        Path(out).parent.mkdir(parents=True, exist_ok=True)
        Path(out).write_text(json.dumps(_PARITY_RECORDS, indent=1))
