"""pytest configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on a CPU-only host: oracle-vs-golden checks, host logic,
the blob layout, and that the C-ABI library loads and exports every symbol the
header declares.  ``-m gpu`` runs the parity tests proper on a B200 through the
C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def q3():
    """The product package (``qwen3-tile-ops_b200``) imported as ``q3b200``."""
    import __graft_entry__ as ge
    return ge.load_package()
