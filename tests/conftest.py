"""Shared pytest setup.

Markers:
  gpu -- needs a CUDA device (B200); run with `pytest -m gpu`.
Everything else runs on a CPU-only machine.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
