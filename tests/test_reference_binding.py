"""The reference's own Python binding (python/omni_tokenizer/native.py of the
reference checkout) loading libomni_b200.so as its OMNI_LIBRARY: every
signature it declares binds, and calls that need no device behave as the
reference documents.  CPU only; skipped where the reference checkout is absent
(it never travels to GPU machines)."""

import os
import sys
from pathlib import Path

import pytest

from tests.conftest import REFERENCE, ROOT, load_package

REFERENCE_PY = REFERENCE / "python"


@pytest.fixture()
def native(monkeypatch):
    if not (REFERENCE_PY / "omni_tokenizer" / "native.py").is_file():
        pytest.skip("reference checkout not present")
    monkeypatch.syspath_prepend(str(REFERENCE_PY))
    monkeypatch.setenv("OMNI_LIBRARY", str(ROOT / "omni-tokenizer_b200" / "libomni_b200.so"))
    for name in [m for m in sys.modules if m == "omni_tokenizer" or m.startswith("omni_tokenizer.")]:
        monkeypatch.delitem(sys.modules, name)
    import omni_tokenizer.native as native

    return native


def test_reference_binding_loads_this_library(native, tmp_path):
    lib = native.Library()  # binds every omni_* signature the reference declares
    assert Path(lib.path) == (ROOT / "omni-tokenizer_b200" / "libomni_b200.so").resolve()
    assert lib.lib.omni_version().startswith(b"0.1.0")
    load_package()
    import omni_tokenizer_b200.omnivq as ov

    path = tmp_path / "tiny.omni"
    ov.write_random_model(path, ov.image_config(layers=1, width=16, heads=2, ffn=32, patch=4, grid=2,
                                                code_dim=8, vocab=16), seed=3)
    with pytest.raises(native.NativeError) as e:  # this library has no CPU backend
        native.Model(lib, path, "cpu")
    assert e.value.status == 4 and "CUDA" in str(e.value)
    if not lib.lib.omni_has_cuda():
        with pytest.raises(native.NativeError):
            native.Model(lib, path, "cuda:0")
