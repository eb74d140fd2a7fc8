"""CPU-side checks of the C ABI: the library builds, loads without a GPU and
exports every entry point include/omni_b200.h declares; argument errors are
reported through omni_b200_last_error() without touching a device."""

import ctypes as C
import re
from pathlib import Path

import pytest

from tests.conftest import ROOT, load_package

HEADER = ROOT / "include" / "omni_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"OMNI_B200_API\s+[\w\s\*]+?\b(omni_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "omni_b200_attention_bhld" in names and "omni_b200_vq_argmin" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol():
    pkg = load_package()
    lib = pkg.library()  # raises if any bound symbol is missing
    for name in declared_symbols():
        assert hasattr(lib.lib, name), name
    assert lib.version().startswith("0.1.0")


def test_argument_errors_need_no_device():
    lib = load_package().library()
    st = lib.lib.omni_b200_attention_bhld(None, None, None, None, 1, 1, 1, 64, 1, 1, None, 0, 0, 0.0, None)
    assert st == 1 and b"null" in lib.lib.omni_b200_last_error()
    st = lib.lib.omni_b200_vq_argmin(None, None, None, None, 1, 64, 10, 1, 1, None, 0, None)
    assert st == 1
    handle = C.c_void_p()
    st = lib.lib.omni_b200_context_create(0, C.byref(handle))
    # Without a GPU the context cannot be created: UNSUPPORTED, never a crash.
    import torch

    if not torch.cuda.is_available():
        assert st == 4 and not handle
    else:
        lib.lib.omni_b200_context_free(handle)


def test_workspace_queries():
    lib = load_package().library()
    # bf16 head-major rows of 72-wide heads need no repacking; fp32 rows do.
    assert lib.lib.omni_b200_attention_rows_workspace(729, 16, 72, 1, 0) == 0
    assert lib.lib.omni_b200_attention_rows_workspace(1500, 20, 64, 0, 0) >= 3 * 20 * 1500 * 64 * 2
    assert lib.lib.omni_b200_vq_workspace(1000, 64, 16384, 1) >= 8000
