"""The one-process multi-GPU host driver (omni-tokenizer_b200/multidevice.py):
split and reassembly logic with stand-in sessions (CPU only)."""

import threading

import numpy as np

from tests.conftest import load_package


class FakeSession:
    """Codes that identify the item: every code of item i is pixels[i, 0, 0, 0]
    (images) or mel[i, 0, 0] (audio)."""

    def __init__(self, device, log):
        self.device, self.log = device, log

    def encode_images(self, pixels, patch):
        self.log.append((self.device, threading.get_ident(), pixels.shape[0]))
        per = (pixels.shape[2] // patch) * (pixels.shape[3] // patch)
        return np.repeat(pixels[:, 0, 0, 0].astype(np.uint16), per)

    def encode_audio_batch(self, mel, valid):
        self.log.append((self.device, threading.get_ident(), mel.shape[0]))
        return np.concatenate([np.full((int(v) + 7) // 8, mel[i, 0, 0], np.uint16) for i, v in enumerate(valid)])

    def close(self):
        pass


def _encoder(devices, log):
    load_package()
    from omni_tokenizer_b200.multidevice import MultiDeviceEncoder

    return MultiDeviceEncoder(devices, lambda d: FakeSession(d, log))


def test_images_split_evenly_and_reassemble_in_order():
    log = []
    with _encoder([0, 1, 2], log) as enc:
        px = np.zeros((10, 3, 16, 8), np.float32)
        px[:, 0, 0, 0] = np.arange(10) + 100
        codes = enc.encode_images(px, patch=4)
    assert codes.shape == (10, 8)
    assert np.array_equal(codes, np.repeat(np.arange(100, 110, dtype=np.uint16)[:, None], 8, 1))
    assert sorted(n for _, _, n in log) == [3, 3, 4]


def test_audio_balanced_bins_and_per_item_codes():
    log = []
    valid = [3000, 100, 2999, 808, 8, 1500, 2200]
    mel = np.zeros((len(valid), 4, 3000), np.float32)
    mel[:, 0, 0] = np.arange(len(valid)) + 7
    with _encoder([0, 1], log) as enc:
        codes = enc.encode_audio(mel, valid)
    assert len(codes) == len(valid)
    for i, (c, v) in enumerate(zip(codes, valid)):
        assert c.shape == ((v + 7) // 8,) and np.all(c == i + 7)
    from omni_tokenizer_b200.sharding import balanced_bins

    assert sorted(n for _, _, n in log) == sorted(len(b) for b in balanced_bins(valid, 2))


def test_fewer_items_than_devices():
    log = []
    with _encoder([0, 1, 2, 3], log) as enc:
        px = np.zeros((2, 3, 8, 8), np.float32)
        px[:, 0, 0, 0] = [5, 9]
        codes = enc.encode_images(px, patch=8)
    assert codes.ravel().tolist() == [5, 9]
    assert len(log) == 2
