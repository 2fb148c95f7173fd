"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on a CPU-only machine (oracle vs golden fixtures, host-side
logic, C-ABI symbol checks, gloo multi-rank tests); ``-m gpu`` needs a B200 and the
built CUDA library.
"""
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "mlsys-flashlinfer-contest_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")
