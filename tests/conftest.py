"""Test configuration: import paths, the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on a machine without a GPU (oracle pins, option logic, host logic, the
C-ABI exports).  ``-m gpu`` tests call the CUDA library through its C ABI on a B200.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "pov-shuffle_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_api():
    from oracle import api

    api.lib()
    return api


@pytest.fixture(scope="session")
def golden_numpy_path():
    data = np.load(GOLDEN / "numpy_path_golden.npz")
    cases = []
    for key in data["cases"]:
        key = str(key)
        n_rows, P, V, iters, seed = (int(x) for x in data[f"{key}__meta"])
        cases.append(
            dict(
                name=key,
                input=data[f"{key}__input"],
                output=data[f"{key}__output"],
                n_rows=n_rows,
                P=P,
                V=V,
                iterations=iters,
                seed=seed,
                offsets=[int(x) for x in data[f"{key}__offsets"]],
            )
        )
    return cases
