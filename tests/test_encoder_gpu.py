"""The reference's outer C ABI on B200 (libomni_b200.so, include/omni_abi.h):
whole audio and image encoder graphs against the reference's own CPU library
(golden fixtures from tests/golden/encoder/make_encoder_golden.py; a live
check when oracle/_ref/libomni_ref_full.so is present), plus the C API
behaviours of omni-tokenizer src/runtime.cpp:131-288 that need a device.

Tolerances: audio (fp32 profile) features within 1e-4 of the reference's fp32
values, image (bf16 profile) features within 1/128 (the reference's own
CUDA-vs-fixture tolerance, tests/test_native.py:55-58).  Codes: (1) this
library's codes are exactly the oracle VQ of this library's features (ties
aside: the BASELINE top-2 rule); (2) a code that differs from the reference's
is one whose distance to the reference's features is within the bound the
measured feature difference allows (|d(f, c) - d(f', c)| <= 2 |f - f'| |c| +
| |f|^2 - |f'|^2 |), plus bf16 rounding of the distance.
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import ROOT, load_package

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "encoder"


@pytest.fixture(scope="module")
def abi():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    load_package()
    import omni_tokenizer_b200.abi as abi

    return abi


@pytest.fixture(scope="module")
def ours(abi):
    import os

    path = os.environ.get("OMNI_B200_LIBRARY") or str(ROOT / "omni-tokenizer_b200" / "libomni_b200.so")
    return abi.OmniLib(path)


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN / "golden.npz"))


def _codebook(kind):
    load_package()
    import omni_tokenizer_b200.omnivq as ov
    from tests.golden.encoder.make_encoder_golden import AUDIO_CFG, IMAGE_CFG

    if kind == "audio":
        cfg = ov.audio_config(**AUDIO_CFG)
        cb = ov.random_tensors(cfg, seed=11)["codebook.weight"]
    else:
        cfg = ov.image_config(**IMAGE_CFG)
        cb = O.round_bf16(ov.random_tensors(cfg, seed=12)["quantize.embedding.weight"])
        cb = cb / np.maximum(O.round_bf16(np.sqrt((cb * cb).sum(1, keepdims=True))), O.round_bf16(np.float32(1e-12)))
        cb = O.round_bf16(cb)
    return cb


def _check_codes(got, want, ours, ref, cb, bf16):
    # (1) Our codes are the oracle VQ of our own features.
    own = O.quantize(ours, cb, bf16=bf16).astype(np.int64)
    mism = np.nonzero(got != own)[0]
    if len(mism):
        d1, d2 = O.quantize_top2(ours[mism], cb, bf16=bf16)
        assert np.all((d2 - d1) < 1e-3 * np.abs(d1)), f"VQ of our features differs at rows {mism}"
    # (2) Differences from the reference stay within the feature-difference bound.
    mism = np.nonzero(got != want)[0]
    f, g = ref.astype(np.float64), ours.astype(np.float64)
    c = cb.astype(np.float64)
    cmax = np.sqrt((c * c).sum(1)).max()
    for r in mism:
        d_want = ((f[r] - c[want[r]]) ** 2).sum()
        d_got = ((f[r] - c[got[r]]) ** 2).sum()
        delta = np.sqrt(((f[r] - g[r]) ** 2).sum())
        slack = 2 * (2 * delta * cmax + abs((f[r] ** 2).sum() - (g[r] ** 2).sum()))
        slack += (2.0 ** -6) * (abs(d_want) + 1.0) if bf16 else 1e-6 * (abs(d_want) + 1.0)
        assert d_got - d_want <= slack, (r, d_got, d_want, slack)


def test_audio_encoder_matches_reference(abi, ours, golden):
    cb = _codebook("audio")
    with ours.load(GOLDEN / "audio.omni", backend=abi.CUDA) as m:
        info = m.info()
        assert (info.kind, info.layers, info.width, info.backend) == (1, 2, 32, 1)
        s = m.context()
        for i in range(3):
            mel, valid = golden[f"audio{i}_mel"], int(golden[f"audio{i}_valid"])
            codes = s.encode_audio(mel, valid)
            feats = s.features(len(codes))
            want = golden[f"audio{i}_features"]
            assert feats.shape == want.shape
            np.testing.assert_allclose(feats, want, rtol=1e-4, atol=1e-4)
            _check_codes(codes.astype(np.int64), golden[f"audio{i}_codes"].astype(np.int64), feats, want, cb, False)
        assert s.peak_workspace > 0
        s.close()


def test_image_encoder_matches_reference(abi, ours, golden):
    cb = _codebook("image")
    with ours.load(GOLDEN / "image.omni", backend=abi.CUDA) as m:
        s = m.context()
        for i in range(3):
            px = golden[f"image{i}_pixels"]
            codes = s.encode_image(px)
            feats = s.features(len(codes))
            want = golden[f"image{i}_features"]
            assert feats.shape == want.shape
            assert np.abs(feats - want).max() <= 1 / 128
            _check_codes(codes.astype(np.int64), golden[f"image{i}_codes"].astype(np.int64), feats, want, cb, True)
        s.close()


def test_batched_audio_matches_per_item_reference(abi, ours, golden):
    """omni_b200_encode_audio_batch: segments of one frame count with different
    valid lengths equal the reference run segment by segment."""
    cb = _codebook("audio")
    mels, valid = golden["audio_batch_mel"], golden["audio_batch_valid"]
    want_codes, want = golden["audio_batch_codes"].astype(np.int64), golden["audio_batch_features"]
    with ours.load(GOLDEN / "audio.omni") as m:
        s = m.context()
        codes = s.encode_audio_batch(mels, valid)
        feats = s.features(len(codes))
        assert feats.shape == want.shape
        np.testing.assert_allclose(feats, want, rtol=1e-4, atol=1e-4)
        _check_codes(codes.astype(np.int64), want_codes, feats, want, cb, False)
        # Device-resident input gives the same codes.
        dev = torch.from_numpy(mels).cuda()
        again = s.encode_audio_batch(tuple(dev.shape), valid, device_ptr=dev.data_ptr())
        np.testing.assert_array_equal(again, codes)
        s.close()


def test_batched_images_match_per_item_reference(abi, ours, golden):
    cb = _codebook("image")
    pxs = golden["image_batch_pixels"]
    want_codes, want = golden["image_batch_codes"].astype(np.int64), golden["image_batch_features"]
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        codes = s.encode_images(pxs, patch=8)
        feats = s.features(len(codes))
        assert feats.shape == want.shape
        assert np.abs(feats - want).max() <= 1 / 128
        _check_codes(codes.astype(np.int64), want_codes, feats, want, cb, True)
        dev = torch.from_numpy(pxs).cuda()
        again = s.encode_images(tuple(dev.shape), patch=8, device_ptr=dev.data_ptr())
        np.testing.assert_array_equal(again, codes)
        # Non-finite input anywhere in the batch fails the call.
        bad = pxs.copy()
        bad[3, 1, 5, 7] = np.inf
        with pytest.raises(abi.OmniError) as e:
            s.encode_images(bad, patch=8)
        assert e.value.status == 1 and "non-finite" in str(e.value)
        s.close()


def test_batched_images_across_chunks(abi, ours):
    """A batch larger than one chunk (host input double-buffered through the
    copy stream) equals the same images sent in single-chunk pieces."""
    rng = np.random.default_rng(91)
    pxs = rng.uniform(-1, 1, (20000, 3, 32, 24)).astype(np.float32)  # 12 rows per image: 3 chunks
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        whole = s.encode_images(pxs, patch=8)
        whole_f = s.features(len(whole))
        parts, parts_f = [], []
        for i in range(0, len(pxs), 5000):
            parts.append(s.encode_images(pxs[i:i + 5000], patch=8))
            parts_f.append(s.features(len(parts[-1])))
        parts, parts_f = np.concatenate(parts), np.concatenate(parts_f)
        assert np.abs(whole_f - parts_f).max() <= 1 / 128
        _check_codes(whole.astype(np.int64), parts.astype(np.int64), whole_f, parts_f, _codebook("image"), True)
        s.close()


_EMULATED_PROBE = r"""
import sys, json
import numpy as np
sys.path.insert(0, sys.argv[1])
from tests.conftest import load_package
load_package()
import omni_tokenizer_b200.abi as abi
lib = abi.OmniLib(sys.argv[2])
import ctypes, os
emulated = hasattr(ctypes.CDLL("libcublas.so.12", mode=os.RTLD_LAZY | os.RTLD_NOLOAD), "cublasSetEmulationStrategy")
g = dict(np.load(sys.argv[3]))
out = {"emulated": np.array(emulated)}
with lib.load(sys.argv[4]) as m:
    s = m.context()
    for i in range(3):
        codes = s.encode_audio(g[f"audio{i}_mel"], int(g[f"audio{i}_valid"]))
        out[f"codes{i}"], out[f"features{i}"] = codes, s.features(len(codes))
    codes = s.encode_audio_batch(g["audio_batch_mel"], g["audio_batch_valid"])
    out["codes_batch"], out["features_batch"] = codes, s.features(len(codes))
    s.close()
np.savez(sys.argv[5], **out)
"""


def test_audio_fp32_emulation_matches_reference(abi, ours, golden, tmp_path):
    """In a process without torch this library's own cuBLAS (with BF16x9 fp32
    emulation) is bound, and fp32-profile GEMMs run emulated: features stay
    within the fp32 tolerance of the reference."""
    import subprocess
    import sys

    lib_path = ours.path
    out = tmp_path / "emulated.npz"
    subprocess.run([sys.executable, "-c", _EMULATED_PROBE, str(ROOT), lib_path, str(GOLDEN / "golden.npz"),
                    str(GOLDEN / "audio.omni"), str(out)], check=True, timeout=300)
    got = dict(np.load(out))
    if not bool(got["emulated"]):
        pytest.skip("the toolkit's cuBLAS has no fp32 emulation")
    cb = _codebook("audio")
    for i in range(3):
        want = golden[f"audio{i}_features"]
        np.testing.assert_allclose(got[f"features{i}"], want, rtol=1e-4, atol=1e-4)
        _check_codes(got[f"codes{i}"].astype(np.int64), golden[f"audio{i}_codes"].astype(np.int64),
                     got[f"features{i}"], want, cb, False)
    np.testing.assert_allclose(got["features_batch"], golden["audio_batch_features"], rtol=1e-4, atol=1e-4)


def test_audio_bf16_mode_matches_graph_oracle(abi, ours, golden, monkeypatch):
    """OMNI_B200_AUDIO_BF16=1: the audio graph in bf16 (bf16 weights and
    activations, the reference's bf16 rounding points) against the numpy graph
    restatement in the same profile (oracle/encoder.py, itself pinned to the
    reference's fixtures).  Summation orders differ, so a rounded intermediate
    may land one bf16 ulp apart: features within 4 ulps of the largest
    feature, on average within a quarter ulp."""
    from oracle import encoder as E

    model = E.load_model(GOLDEN / "audio.omni")
    cb = _codebook("audio")
    monkeypatch.setenv("OMNI_B200_AUDIO_BF16", "1")
    with ours.load(GOLDEN / "audio.omni") as m:
        s = m.context()
        cases = [(golden[f"audio{i}_mel"][None], [int(golden[f"audio{i}_valid"])]) for i in range(3)]
        cases.append((golden["audio_batch_mel"], list(golden["audio_batch_valid"])))
        for mels, valid in cases:
            codes = s.encode_audio_batch(mels, valid)
            feats = s.features(len(codes))
            want = np.concatenate([E.audio(model, mel, v, bf16=True)[1] for mel, v in zip(mels, valid)])
            assert feats.shape == want.shape
            ulp = 2.0 ** (np.floor(np.log2(np.abs(want).max())) - 7)
            diff = np.abs(feats - want)
            assert diff.max() <= 4 * ulp and diff.mean() <= 0.25 * ulp, (diff.max(), diff.mean(), ulp)
            want_codes = O.quantize(want, cb, O.squares(cb)).astype(np.int64)
            _check_codes(codes.astype(np.int64), want_codes, feats, want, cb, False)
        s.close()


def test_live_reference_cross_check(abi, ours):
    """Same inputs through the reference CPU library (when built) and this library."""
    ref_path = ROOT / "oracle" / "_ref" / "libomni_ref_full.so"
    if not ref_path.is_file():
        pytest.skip("reference CPU library not built")
    ref = abi.OmniLib(ref_path)
    rng = np.random.default_rng(77)
    px = rng.uniform(-1, 1, (3, 40, 24)).astype(np.float32)
    with ref.load(GOLDEN / "image.omni", backend=abi.CPU) as rm, ours.load(GOLDEN / "image.omni") as om:
        rs, os_ = rm.context(), om.context()
        want, got = rs.encode_image(px), os_.encode_image(px)
        wf, gf = rs.features(len(want)), os_.features(len(got))
        assert np.abs(wf - gf).max() <= 1 / 128
        _check_codes(got.astype(np.int64), want.astype(np.int64), gf, wf, _codebook("image"), True)
        rs.close(), os_.close()


def test_api_behaviour(abi, ours, golden):
    lib = ours.lib
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        # No features before the first encode.
        count = C.c_size_t()
        buf = np.zeros(4, np.float32)
        assert lib.omni_context_copy_features(s.handle, buf.ctypes.data_as(C.POINTER(C.c_float)), 4, C.byref(count)) == 1
        # Size query: NULL codes, zero capacity -> INVALID_ARGUMENT with the count.
        px = golden["image1_pixels"]
        assert lib.omni_encode_image(s.handle, px.ctypes.data_as(C.POINTER(C.c_float)), 48, 32, None, 0,
                                     C.byref(count)) == 1
        assert count.value == 24
        assert b"capacity is too small" in lib.omni_last_error()
        # Cancel -> CANCELLED; reset -> works again.
        s.cancel()
        with pytest.raises(abi.OmniError) as e:
            s.encode_image(px)
        assert e.value.status == 6
        s.reset_cancel()
        assert s.encode_image(px).size == 24
        # Trace callback: the reference's image stage names.
        stages = []

        def cb(user, stage, values, rows, cols):
            stages.append((stage.decode(), rows, cols))

        fn = abi.TRACE(cb)
        assert lib.omni_context_set_trace(s.handle, fn, None) == 0
        s.encode_image(golden["image0_pixels"])
        names = [n for n, _, _ in stages]
        assert names == ["patch", "position", "embedding", "norm1.0", "qkv.0", "attention.0", "residual1.0",
                         "fc1.0", "gelu.0", "fc2.0", "layer.0", "layer.1", "projected"]
        assert stages[4][1:] == (16, 96)
        # Non-finite input -> INVALID_ARGUMENT.
        bad = golden["image0_pixels"].copy()
        bad[0, 0, 0] = np.nan
        with pytest.raises(abi.OmniError) as e:
            s.encode_image(bad)
        assert e.value.status == 1
        s.close()
    # Invalid model files.
    with pytest.raises(abi.OmniError) as e:
        ours.load(GOLDEN / "no_such_model.omni")
    assert e.value.status == 2
    with pytest.raises(abi.OmniError) as e:
        ours.load(GOLDEN / "golden.npz")
    assert e.value.status == 3


def test_plain_cublas_fallback_matches_reference(abi, ours, golden, monkeypatch):
    """OMNI_B200_CUBLASLT=0: linears as plain cuBLAS GEMMs plus the separate
    bias / rounding epilogue kernel -- the same results within the tolerances."""
    monkeypatch.setenv("OMNI_B200_CUBLASLT", "0")
    cb = _codebook("image")
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        for i in range(3):
            codes = s.encode_image(golden[f"image{i}_pixels"])
            feats = s.features(len(codes))
            want = golden[f"image{i}_features"]
            assert np.abs(feats - want).max() <= 1 / 128
            _check_codes(codes.astype(np.int64), golden[f"image{i}_codes"].astype(np.int64), feats, want, cb, True)
        s.close()
    with ours.load(GOLDEN / "audio.omni") as m:
        s = m.context()
        codes = s.encode_audio_batch(golden["audio_batch_mel"], golden["audio_batch_valid"])
        np.testing.assert_allclose(s.features(len(codes)), golden["audio_batch_features"], rtol=1e-4, atol=1e-4)
        s.close()


def test_concurrent_contexts_share_a_model(abi, ours):
    """Several host threads, one context each on one shared model, encoding at
    the same time: each gets the codes a lone call gets."""
    import threading

    rng = np.random.default_rng(5)
    batches = [rng.uniform(-1, 1, (6, 3, 32, 24)).astype(np.float32) for _ in range(4)]
    with ours.load(GOLDEN / "image.omni") as m:
        lone = []
        for b in batches:
            s = m.context()
            lone.append(s.encode_images(b, patch=8))
            s.close()
        got = [None] * len(batches)
        errors = []

        def work(k):
            try:
                s = m.context()
                for _ in range(3):
                    got[k] = s.encode_images(batches[k], patch=8)
                s.close()
            except Exception as e:  # reported below
                errors.append(e)

        threads = [threading.Thread(target=work, args=(k,)) for k in range(len(batches))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        assert not errors, errors
        for a, b in zip(got, lone):
            np.testing.assert_array_equal(a, b)


def test_two_devices_in_one_process(abi, ours, golden):
    """A model and context per device in one process (kernel attributes and the
    GELU table are per device): both devices give the same codes."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    px = golden["image_batch_pixels"]
    out = []
    for dev in (0, 1):
        with ours.load(GOLDEN / "image.omni", device=dev) as m:
            s = m.context()
            out.append((s.encode_images(px, patch=8), s.features()))
            s.close()
    np.testing.assert_array_equal(out[0][0], out[1][0])
    np.testing.assert_array_equal(out[0][1], out[1][1])


def test_multi_device_encoder_matches_one_session(abi, ours, golden):
    """omni-tokenizer_b200/multidevice.py over every visible device (one thread
    and context each) returns the codes of a single batched call, in order."""
    load_package()
    from omni_tokenizer_b200.multidevice import MultiDeviceEncoder

    devices = list(range(min(torch.cuda.device_count(), 4)))
    rng = np.random.default_rng(17)
    px = rng.uniform(-1, 1, (9, 3, 32, 24)).astype(np.float32)
    mels, valid = golden["audio_batch_mel"], golden["audio_batch_valid"]
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        want_img = s.encode_images(px, patch=8).reshape(9, -1)
        s.close()
    with ours.load(GOLDEN / "audio.omni") as m:
        s = m.context()
        want_audio = [s.encode_audio_batch(mel[None], [v]) for mel, v in zip(mels, valid)]
        s.close()
    with MultiDeviceEncoder(devices, lib=ours, model_path=GOLDEN / "image.omni") as enc:
        np.testing.assert_array_equal(enc.encode_images(px, patch=8), want_img)
    with MultiDeviceEncoder(devices, lib=ours, model_path=GOLDEN / "audio.omni") as enc:
        for got, want in zip(enc.encode_audio(mels, valid), want_audio):
            np.testing.assert_array_equal(got, want)


def test_repeated_batches_replay_a_cuda_graph(abi, ours, golden, monkeypatch):
    """A batched call that repeats (same key, device or page-locked host input,
    no trace callback) is captured on its second call and replayed afterwards.
    The replay recomputes everything from the input: new data in the same
    buffer gives that data's codes, bit-identical to an eager context's."""
    monkeypatch.setenv("OMNI_B200_GRAPHS", "0")
    with ours.load(GOLDEN / "audio.omni") as m:
        eager = m.context()
        monkeypatch.setenv("OMNI_B200_GRAPHS", "1")
        s = m.context()
        mels, valid = golden["audio_batch_mel"], golden["audio_batch_valid"]
        dev = torch.from_numpy(mels).cuda()
        want = eager.encode_audio_batch(mels, valid)
        want_f = eager.features(len(want))
        for i in range(4):
            got = s.encode_audio_batch(tuple(dev.shape), valid, device_ptr=dev.data_ptr())
            np.testing.assert_array_equal(got, want)
            np.testing.assert_array_equal(s.features(len(got)), want_f)
        assert s.graph_launches == 3  # captured on the second call, replayed twice
        assert eager.graph_launches == 0
        # Other data in the same buffer: the replay follows the input.
        other = np.ascontiguousarray(mels[::-1])
        dev.copy_(torch.from_numpy(other))
        got = s.encode_audio_batch(tuple(dev.shape), valid, device_ptr=dev.data_ptr())
        assert s.graph_launches == 4
        np.testing.assert_array_equal(got, eager.encode_audio_batch(other, valid))
        np.testing.assert_array_equal(s.features(len(got)), eager.features(len(got)))
        # A cancellation before a replay: OMNI_CANCELLED, then the replay works again.
        s.cancel()
        with pytest.raises(abi.OmniError) as e:
            s.encode_audio_batch(tuple(dev.shape), valid, device_ptr=dev.data_ptr())
        assert e.value.status == 6
        s.reset_cancel()
        np.testing.assert_array_equal(s.encode_audio_batch(tuple(dev.shape), valid, device_ptr=dev.data_ptr()),
                                      got)
        # Page-locked host input is captured too; pageable host input stays eager.
        pinned = torch.from_numpy(mels).pin_memory()
        before = s.graph_launches
        for _ in range(3):
            np.testing.assert_array_equal(s.encode_audio_batch(pinned.numpy(), valid), want)
        assert s.graph_launches == before + 2
        before = s.graph_launches
        for _ in range(3):
            np.testing.assert_array_equal(s.encode_audio_batch(mels, valid), want)
        assert s.graph_launches == before
        s.close()
        eager.close()
    with ours.load(GOLDEN / "image.omni") as m:
        monkeypatch.setenv("OMNI_B200_GRAPHS", "0")
        eager = m.context()
        monkeypatch.setenv("OMNI_B200_GRAPHS", "1")
        s = m.context()
        pxs = golden["image_batch_pixels"]
        dev = torch.from_numpy(pxs).cuda()
        want = eager.encode_images(pxs, patch=8)
        want_f = eager.features(len(want))
        for _ in range(3):
            got = s.encode_images(tuple(dev.shape), patch=8, device_ptr=dev.data_ptr())
            np.testing.assert_array_equal(got, want)
            np.testing.assert_array_equal(s.features(len(got)), want_f)
        assert s.graph_launches == 2
        s.close()
        eager.close()
