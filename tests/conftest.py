"""Test configuration: import paths and the ``gpu`` marker.

The package directory mirrors the reference's module layout (``backend``,
``comm``, ``contracts``, ``graph``, ``memory``, ``runtime``), so it is put on
``sys.path`` the way the reference's tests put their repository root there.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "flagos-pim-compiler_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
