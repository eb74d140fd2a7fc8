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
    # bf16 rows of 72-wide heads and fp32 rows of 64-wide heads are read in
    # place; fp32 heads of 7 (28-byte rows) are repacked to fp32 [heads, n, 32].
    # 16-bit rows whose (query block, head) items leave the last round of SMs
    # mostly empty get key split scratch: 4 heads x 5 blocks of 1200 rows are 20
    # items (7 parts of 1-2 of the 10 KV tiles).  16 x 3 blocks of 729 rows (48
    # items of 6 tiles) would save 4 tiles, below what the combine pass costs;
    # 16 x 6 blocks of 1500 rows are 96 items (a part would need a second round).
    sms = 148  # the SM count without a device
    assert lib.lib.omni_b200_attention_rows_workspace(1200, 4, 72, 1, 0) >= sms * 256 * (80 + 2) * 4
    assert lib.lib.omni_b200_attention_rows_workspace(729, 16, 72, 1, 0) == 0
    assert lib.lib.omni_b200_attention_rows_workspace(1500, 16, 64, 1, 0) == 0
    assert lib.lib.omni_b200_attention_rows_batch_workspace(1500, 1, 16, 64, 1, 0) == 0
    assert lib.lib.omni_b200_attention_rows_batch_workspace(1500, 2, 16, 64, 1, 1) >= sms * 256 * 66 * 4
    assert lib.lib.omni_b200_attention_rows_batch_workspace(1500, 2, 16, 64, 0, 1) == 0  # fp32: no split
    assert lib.lib.omni_b200_attention_rows_workspace(1500, 20, 64, 0, 0) == 0
    assert lib.lib.omni_b200_attention_rows_workspace(129, 2, 7, 0, 0) >= 3 * 2 * 129 * 32 * 4
    assert lib.lib.omni_b200_attention_rows_workspace(129, 2, 7, 1, 0) >= 3 * 2 * 129 * 16 * 2
    assert lib.lib.omni_b200_vq_workspace(1000, 64, 16384, 1) >= 8000


# ------------------------------------------------ the reference's outer C ABI
ABI_HEADER = ROOT / "include" / "omni_abi.h"


def abi_symbols():
    return sorted(set(re.findall(r"OMNI_ABI_API\s+[\w\s\*]+?\b(omni_\w+)\s*\(", ABI_HEADER.read_text())))


def test_outer_abi_declares_and_exports_the_15_entry_points():
    load_package()
    import omni_tokenizer_b200.abi as abi

    names = abi_symbols()
    assert names == sorted(abi.SYMBOLS + abi.EXTENSION_SYMBOLS) and len(abi.SYMBOLS) == 15
    assert all(n.startswith("omni_b200_") for n in abi.EXTENSION_SYMBOLS)
    lib = abi.OmniLib(ROOT / "omni-tokenizer_b200" / "libomni_b200.so")  # binds all 15 and the extension
    assert lib.batched
    assert lib.lib.omni_version().startswith(b"0.1.0")


def test_batched_extension_argument_errors_without_a_device():
    load_package()
    import omni_tokenizer_b200.abi as abi

    lib = abi.OmniLib(ROOT / "omni-tokenizer_b200" / "libomni_b200.so")
    count = C.c_size_t(7)
    valid = (C.c_uint32 * 1)(8)
    assert lib.lib.omni_b200_encode_audio_batch(None, None, 1, 8, valid, None, 0, C.byref(count)) == 1
    assert b"Invalid audio pointers" in lib.lib.omni_last_error()
    assert lib.lib.omni_b200_encode_images(None, None, 1, 8, 8, None, 0, C.byref(count)) == 1
    assert b"Invalid image pointers" in lib.lib.omni_last_error()


def test_outer_abi_errors_without_a_device(tmp_path):
    load_package()
    import omni_tokenizer_b200.abi as abi
    import omni_tokenizer_b200.omnivq as ov

    lib = abi.OmniLib(ROOT / "omni-tokenizer_b200" / "libomni_b200.so")
    path = tmp_path / "tiny.omni"
    ov.write_random_model(path, ov.image_config(layers=1, width=16, heads=2, ffn=32, patch=4, grid=2,
                                                code_dim=8, vocab=16), seed=3)
    with pytest.raises(abi.OmniError) as e:  # only the CUDA backend exists here
        lib.load(path, backend=abi.CPU)
    assert e.value.status == 4
    handle = C.c_void_p()
    assert lib.lib.omni_model_load(str(path).encode(), abi.CUDA, 0, None) == 1
    assert lib.lib.omni_model_get_info(None, None) == 1
    assert lib.lib.omni_context_create(None, C.byref(handle)) == 1 and not handle
    assert lib.lib.omni_context_peak_workspace(None) == 0
    lib.lib.omni_context_cancel(None)  # no-ops on NULL, like the reference
    lib.lib.omni_model_free(None)
    if not lib.lib.omni_has_cuda():
        with pytest.raises(abi.OmniError) as e:
            lib.load(path)
        assert e.value.status == 4


def test_model_writer_round_trips_through_the_reference_loader(tmp_path):
    """omnivq.write_model output is accepted by the reference's own loader (when built)."""
    ref = ROOT / "oracle" / "_ref" / "libomni_ref_full.so"
    if not ref.is_file():
        pytest.skip("reference CPU library not built")
    load_package()
    import omni_tokenizer_b200.abi as abi
    import omni_tokenizer_b200.omnivq as ov

    lib = abi.OmniLib(ref)
    for cfg in (ov.audio_config(layers=1, width=16, heads=2, ffn=32, mel=8, positions=16, block=8, vocab=32),
                ov.image_config(layers=1, width=16, heads=2, ffn=32, patch=4, grid=2, code_dim=8, vocab=32)):
        path = tmp_path / f"m{cfg.kind}.omni"
        ov.write_random_model(path, cfg, seed=cfg.kind)
        with lib.load(path, backend=abi.CPU) as m:
            info = m.info()
            assert (info.kind, info.layers, info.width, info.code_dim) == (cfg.kind, 1, 16, cfg.code_dim)
