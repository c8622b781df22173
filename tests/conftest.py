"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any machine (oracle vs golden fixtures, host logic, C-ABI
exports and argument validation, gloo multi-process tests). ``-m gpu`` runs the parity
tests of the CUDA kernels through the C ABI on a compute capability 10.0 device.
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "tests", ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (compute capability 10.0) GPU")
