"""Generate the encoder-graph golden fixtures (run where the reference builds).

    make -C oracle ref && python tests/golden/encoder/make_encoder_golden.py

Writes two small seeded OMNIVQ01 models (tests/golden/encoder/audio.omni,
image.omni) with omni_tokenizer_b200.omnivq and runs them on the
reference's own CPU library (oracle/_ref/libomni_ref_full.so, the reference's
src/cpu.cpp + model.cpp + runtime.cpp compiled unchanged) through its omni_*
C ABI; the inputs, codes and pre-VQ features go to golden.npz.
"""

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[3]
sys.path.insert(0, str(ROOT))

from tests.conftest import load_package  # noqa: E402

load_package()
import omni_tokenizer_b200.abi as abi  # noqa: E402
import omni_tokenizer_b200.omnivq as ov  # noqa: E402

HERE = Path(__file__).resolve().parent
AUDIO_CFG = dict(layers=2, width=32, heads=2, ffn=64, mel=16, positions=64, block=16, vocab=128)
IMAGE_CFG = dict(layers=2, width=32, heads=2, ffn=64, patch=8, grid=4, code_dim=16, vocab=128)


def main():
    ref = abi.OmniLib(ROOT / "oracle" / "_ref" / "libomni_ref_full.so")
    ov.write_random_model(HERE / "audio.omni", ov.audio_config(**AUDIO_CFG), seed=11)
    ov.write_random_model(HERE / "image.omni", ov.image_config(**IMAGE_CFG), seed=12)
    rng = np.random.default_rng(2024)
    rng_batch = np.random.default_rng(2025)  # the batch fixtures leave the single-item draws unchanged
    out = {}
    with ref.load(HERE / "audio.omni", backend=abi.CPU) as m:
        s = m.context()
        for i, (frames, valid) in enumerate([(64, 56), (128, 128), (32, 9)]):
            mel = rng.uniform(-1.5, 1.5, (AUDIO_CFG["mel"], frames)).astype(np.float32)
            codes = s.encode_audio(mel, valid)
            out[f"audio{i}_mel"] = mel
            out[f"audio{i}_valid"] = np.int32(valid)
            out[f"audio{i}_codes"] = codes
            out[f"audio{i}_features"] = s.features(len(codes))
        # A batch for the batched extension: segments of one frame count with
        # different valid lengths, each run alone through the reference.
        mels = rng_batch.uniform(-1.5, 1.5, (4, AUDIO_CFG["mel"], 64)).astype(np.float32)
        valid = np.array([64, 33, 8, 57], np.int32)
        codes, feats = [], []
        for mel, v in zip(mels, valid):
            codes.append(s.encode_audio(mel, int(v)))
            feats.append(s.features(len(codes[-1])))
        out["audio_batch_mel"], out["audio_batch_valid"] = mels, valid
        out["audio_batch_codes"], out["audio_batch_features"] = np.concatenate(codes), np.concatenate(feats)
        s.close()
    with ref.load(HERE / "image.omni", backend=abi.CPU) as m:
        s = m.context()
        for i, (h, w) in enumerate([(32, 32), (48, 32), (16, 40)]):
            px = rng.uniform(-1, 1, (3, h, w)).astype(np.float32)
            codes = s.encode_image(px)
            out[f"image{i}_pixels"] = px
            out[f"image{i}_codes"] = codes
            out[f"image{i}_features"] = s.features(len(codes))
        pxs = rng_batch.uniform(-1, 1, (5, 3, 32, 24)).astype(np.float32)
        codes, feats = [], []
        for px in pxs:
            codes.append(s.encode_image(px))
            feats.append(s.features(len(codes[-1])))
        out["image_batch_pixels"] = pxs
        out["image_batch_codes"], out["image_batch_features"] = np.concatenate(codes), np.concatenate(feats)
        s.close()
    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", {k: v.shape for k, v in out.items() if k.endswith("codes")})


if __name__ == "__main__":
    main()
