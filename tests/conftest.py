"""Shared pytest setup.

Markers:
  gpu -- needs a CUDA device (B200); run with `pytest -m gpu`.
Everything else runs on a CPU-only machine.
"""

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
# The reference checkout, read only by the CPU tests that bind or build from it:
# $OMNI_REFERENCE, else a `reference` directory beside this repository.
REFERENCE = Path(os.environ.get("OMNI_REFERENCE") or ROOT.parent / "reference")
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """Import omni-tokenizer_b200/ as the module `omni_tokenizer_b200`."""
    import importlib.util

    name = "omni_tokenizer_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "omni-tokenizer_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod
