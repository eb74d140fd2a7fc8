"""The numpy restatement of the encoder graphs (oracle/encoder.py) pinned to
the reference's own CPU library: its outputs on the golden inputs against the
fixtures of tests/golden/encoder (made by the reference, see
make_encoder_golden.py).  CPU only."""

from pathlib import Path

import numpy as np
import pytest

from oracle import encoder as E
from oracle import oracle as O
from tests.conftest import load_package

GOLDEN = Path(__file__).resolve().parent / "golden" / "encoder"


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN / "golden.npz"))


def _codes_agree(got, want, feats, cb, bf16):
    mism = np.nonzero(got != want)[0]
    if len(mism):  # only where the reference's own top-2 distances nearly tie
        d1, d2 = O.quantize_top2(feats[mism], cb, bf16=bf16)
        assert np.all((d2 - d1) <= 1e-3 * np.abs(d1) + 1e-6), mism


def test_reader_matches_the_writer():
    load_package()
    import omni_tokenizer_b200.omnivq as ov
    from tests.golden.encoder.make_encoder_golden import AUDIO_CFG, IMAGE_CFG

    cfg, t = E.load_model(GOLDEN / "audio.omni")
    want = ov.random_tensors(ov.audio_config(**AUDIO_CFG), seed=11)
    assert cfg["kind"] == 1 and cfg["width"] == AUDIO_CFG["width"] and set(t) == set(want)
    assert all(np.array_equal(t[n], want[n]) for n in want)
    cfg, t = E.load_model(GOLDEN / "image.omni")
    want = ov.random_tensors(ov.image_config(**IMAGE_CFG), seed=12)
    assert all(np.array_equal(t[n], O.round_bf16(want[n])) for n in want)


def test_audio_graph_matches_reference(golden):
    model = E.load_model(GOLDEN / "audio.omni")
    cb = model[1]["codebook.weight"]
    for i in range(3):
        codes, feats = E.audio(model, golden[f"audio{i}_mel"], int(golden[f"audio{i}_valid"]))
        np.testing.assert_allclose(feats, golden[f"audio{i}_features"], rtol=1e-5, atol=1e-5)
        _codes_agree(codes, golden[f"audio{i}_codes"], feats, cb, False)
    feats = np.concatenate([E.audio(model, m, int(v))[1] for m, v in
                            zip(golden["audio_batch_mel"], golden["audio_batch_valid"])])
    np.testing.assert_allclose(feats, golden["audio_batch_features"], rtol=1e-5, atol=1e-5)


def test_image_graph_matches_reference(golden):
    model = E.load_model(GOLDEN / "image.omni")
    cb = E.normalize(model[1]["quantize.embedding.weight"], True)
    for i in range(3):
        codes, feats = E.image(model, golden[f"image{i}_pixels"])
        assert np.abs(feats - golden[f"image{i}_features"]).max() <= 1 / 128
        _codes_agree(codes, golden[f"image{i}_codes"], feats, cb, True)
