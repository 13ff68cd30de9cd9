"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a CUDA device, run with
  ``pytest -m gpu`` on a B200);
* puts the repository root (for ``oracle``) and ``flash-mhc_b200`` (for the
  ``flash_mhc`` package) on ``sys.path``.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "flash-mhc_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
