"""One process, several GPUs: a host driver over the batched C ABI.

The reference scales by running one Tokenizer per GPU
(python/omni_tokenizer/runtime.py:52-57, ``omni_model_load(..., device=N)``).
``MultiDeviceEncoder`` does that inside one process: it loads the model once per
device, keeps one context per device, and drives each from its own host thread
(the ctypes calls release the GIL, so the devices run concurrently).  A batch
is split with the rules of :mod:`sharding` -- contiguous equal ranges for
images, length-balanced bins (cost L**2 of the valid frames) for audio -- and
the codes are reassembled in input order.  Items are independent, so there is
no exchange between devices on the data path.

Sessions come from ``session_factory(device)``; the default opens
``lib.load(model_path, device=device).context()`` on an :class:`abi.OmniLib`.
Any object with ``encode_images(pixels, patch)`` / ``encode_audio_batch(mel,
valid)`` and ``close()`` works, which keeps the split / reassembly logic
testable without a GPU.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Callable, List, Optional, Sequence

import numpy as np

from .sharding import balanced_bins, even_split


class MultiDeviceEncoder:
    def __init__(self, devices: Sequence[int], session_factory: Optional[Callable[[int], object]] = None, *,
                 lib=None, model_path=None):
        if not devices:
            raise ValueError("at least one device is required")
        self.devices = list(devices)
        self._models = []
        if session_factory is None:
            if lib is None or model_path is None:
                raise ValueError("give session_factory, or lib and model_path")

            def session_factory(device, _lib=lib, _path=model_path):
                model = _lib.load(_path, device=device)
                self._models.append(model)
                return model.context()

        self.sessions = [session_factory(d) for d in self.devices]
        self._pool = ThreadPoolExecutor(max_workers=len(self.devices))

    def close(self):
        self._pool.shutdown(wait=True)
        for s in self.sessions:
            s.close()
        for m in self._models:
            m.close()
        self.sessions, self._models = [], []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _run(self, calls):
        futures = [self._pool.submit(fn) if fn is not None else None for fn in calls]
        return [f.result() if f is not None else None for f in futures]

    def encode_images(self, pixels: np.ndarray, patch: int) -> np.ndarray:
        """pixels [items, 3, h, w] -> codes [items, (h / patch) * (w / patch)] in input order."""
        pixels = np.ascontiguousarray(pixels, np.float32)
        items = pixels.shape[0]
        per_item = (pixels.shape[2] // patch) * (pixels.shape[3] // patch)
        parts = even_split(items, len(self.devices))
        calls = [(lambda s=s, r=r: s.encode_images(pixels[r.start:r.stop], patch)) if len(r) else None
                 for s, r in zip(self.sessions, parts)]
        out = np.zeros((items, per_item), np.uint16)
        for r, codes in zip(parts, self._run(calls)):
            if codes is not None:
                out[r.start:r.stop] = np.asarray(codes).reshape(len(r), per_item)
        return out

    def encode_audio(self, mel: np.ndarray, valid_frames: Sequence[int]) -> List[np.ndarray]:
        """mel [items, mel, frames], valid_frames[items] -> per-item code arrays in input order."""
        mel = np.ascontiguousarray(mel, np.float32)
        valid = np.asarray(valid_frames, np.int64)
        if valid.shape != (mel.shape[0],):
            raise ValueError("one valid frame count per segment")
        bins = balanced_bins([int(v) for v in valid], len(self.devices))
        calls = []
        for s, idx in zip(self.sessions, bins):
            if idx:
                sel = np.asarray(idx)
                calls.append(lambda s=s, sel=sel: s.encode_audio_batch(mel[sel], valid[sel].astype(np.uint32)))
            else:
                calls.append(None)
        out: List[Optional[np.ndarray]] = [None] * mel.shape[0]
        for idx, codes in zip(bins, self._run(calls)):
            if codes is None:
                continue
            counts = [(int(valid[i]) + 7) // 8 for i in idx]
            pieces = np.split(np.asarray(codes), np.cumsum(counts)[:-1])
            for i, piece in zip(idx, pieces):
                out[i] = piece
        return out
