"""ctypes binding of the omni_* C ABI (include/omni_abi.h).

The same 15 entry points as omni-tokenizer's include/omni/omni.h, so this
binding drives libomni_b200.so (CUDA backend) and, in tests and the CPU
baseline, the reference's own CPU library alike.  Errors raise OmniError with
the library's thread-local message, like the reference's native.py.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

CPU, CUDA = 0, 1


class OmniError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"omni status {status}: {message}")
        self.status = status


class ModelInfo(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("kind", C.c_uint32), ("layers", C.c_uint32),
                ("width", C.c_uint32), ("heads", C.c_uint32), ("code_dim", C.c_uint32),
                ("vocabulary_size", C.c_uint32), ("backend", C.c_uint32), ("weight_bytes", C.c_uint64)]


TRACE = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_size_t, C.c_size_t)

_SIGS = {
    "omni_last_error": (C.c_char_p, []),
    "omni_version": (C.c_char_p, []),
    "omni_has_cuda": (C.c_int, []),
    "omni_model_load": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "omni_model_free": (None, [C.c_void_p]),
    "omni_model_get_info": (C.c_int, [C.c_void_p, C.POINTER(ModelInfo)]),
    "omni_context_create": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "omni_context_free": (None, [C.c_void_p]),
    "omni_context_cancel": (None, [C.c_void_p]),
    "omni_context_reset_cancel": (None, [C.c_void_p]),
    "omni_context_set_trace": (C.c_int, [C.c_void_p, TRACE, C.c_void_p]),
    "omni_encode_audio": (C.c_int, [C.c_void_p, C.POINTER(C.c_float), C.c_uint32, C.c_uint32,
                                    C.POINTER(C.c_uint16), C.c_size_t, C.POINTER(C.c_size_t)]),
    "omni_encode_image": (C.c_int, [C.c_void_p, C.POINTER(C.c_float), C.c_uint32, C.c_uint32,
                                    C.POINTER(C.c_uint16), C.c_size_t, C.POINTER(C.c_size_t)]),
    "omni_context_copy_features": (C.c_int, [C.c_void_p, C.POINTER(C.c_float), C.c_size_t,
                                             C.POINTER(C.c_size_t)]),
    "omni_context_peak_workspace": (C.c_uint64, [C.c_void_p]),
}
SYMBOLS = tuple(_SIGS)
# Batched extension of libomni_b200.so (absent from the reference's library).
_EXT_SIGS = {
    "omni_b200_encode_audio_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                               C.POINTER(C.c_uint32), C.POINTER(C.c_uint16), C.c_size_t,
                                               C.POINTER(C.c_size_t)]),
    "omni_b200_encode_images": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                          C.POINTER(C.c_uint16), C.c_size_t, C.POINTER(C.c_size_t)]),
    "omni_b200_context_graph_launches": (C.c_uint64, [C.c_void_p]),
}
EXTENSION_SYMBOLS = tuple(_EXT_SIGS)


class OmniLib:
    def __init__(self, path):
        self.path = str(path)
        self.lib = C.CDLL(self.path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(self.lib, name)
            fn.restype, fn.argtypes = res, args
        self.batched = all(hasattr(self.lib, n) for n in _EXT_SIGS)
        if self.batched:
            for name, (res, args) in _EXT_SIGS.items():
                fn = getattr(self.lib, name)
                fn.restype, fn.argtypes = res, args

    def check(self, status):
        if status:
            raise OmniError(status, self.lib.omni_last_error().decode(errors="replace"))

    def load(self, model_path, backend=CUDA, device=0):
        return Model(self, model_path, backend, device)


class Model:
    def __init__(self, lib: OmniLib, path, backend, device):
        self.lib = lib
        self.handle = C.c_void_p()
        lib.check(lib.lib.omni_model_load(str(path).encode(), backend, device, C.byref(self.handle)))

    def info(self):
        out = ModelInfo(struct_size=C.sizeof(ModelInfo))
        self.lib.check(self.lib.lib.omni_model_get_info(self.handle, C.byref(out)))
        return out

    def context(self):
        return Session(self)

    def close(self):
        if self.handle:
            self.lib.lib.omni_model_free(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Session:
    def __init__(self, model: Model):
        self.lib = model.lib
        self.handle = C.c_void_p()
        self.lib.check(self.lib.lib.omni_context_create(model.handle, C.byref(self.handle)))

    def encode_audio(self, mel, valid_frames):
        mel = np.ascontiguousarray(mel, np.float32)
        frames = mel.shape[1]
        codes = np.zeros((valid_frames + 7) // 8, np.uint16)
        count = C.c_size_t()
        self.lib.check(self.lib.lib.omni_encode_audio(
            self.handle, mel.ctypes.data_as(C.POINTER(C.c_float)), frames, valid_frames,
            codes.ctypes.data_as(C.POINTER(C.c_uint16)), codes.size, C.byref(count)))
        return codes[: count.value]

    def encode_image(self, pixels):
        pixels = np.ascontiguousarray(pixels, np.float32)
        _, h, w = pixels.shape
        count = C.c_size_t()
        status = self.lib.lib.omni_encode_image(self.handle, pixels.ctypes.data_as(C.POINTER(C.c_float)), h, w,
                                                None, 0, C.byref(count))
        if status != 1:  # the size query answers INVALID_ARGUMENT with the count
            self.lib.check(status)
        codes = np.zeros(count.value, np.uint16)
        self.lib.check(self.lib.lib.omni_encode_image(
            self.handle, pixels.ctypes.data_as(C.POINTER(C.c_float)), h, w,
            codes.ctypes.data_as(C.POINTER(C.c_uint16)), codes.size, C.byref(count)))
        return codes

    def encode_audio_batch(self, mel, valid_frames, device_ptr=None):
        """mel [items, mel, frames] fp32 (or device_ptr to the same layout on the
        model's device); returns the concatenated codes."""
        items, _, frames = mel.shape if device_ptr is None else mel
        valid = np.ascontiguousarray(valid_frames, np.uint32)
        codes = np.zeros(int(((valid.astype(np.int64) + 7) // 8).sum()), np.uint16)
        if device_ptr is None:
            mel = np.ascontiguousarray(mel, np.float32)
            ptr = mel.ctypes.data
        else:
            ptr = device_ptr
        count = C.c_size_t()
        self.lib.check(self.lib.lib.omni_b200_encode_audio_batch(
            self.handle, C.c_void_p(ptr), items, frames, valid.ctypes.data_as(C.POINTER(C.c_uint32)),
            codes.ctypes.data_as(C.POINTER(C.c_uint16)), codes.size, C.byref(count)))
        return codes[: count.value]

    def encode_images(self, pixels, patch, device_ptr=None):
        """pixels [items, 3, h, w] fp32 (or, with device_ptr, its shape tuple and
        the device address); returns the codes, image after image."""
        items, _, h, w = pixels.shape if device_ptr is None else pixels
        codes = np.zeros(items * (h // patch) * (w // patch), np.uint16)
        if device_ptr is None:
            pixels = np.ascontiguousarray(pixels, np.float32)
            ptr = pixels.ctypes.data
        else:
            ptr = device_ptr
        count = C.c_size_t()
        self.lib.check(self.lib.lib.omni_b200_encode_images(
            self.handle, C.c_void_p(ptr), items, h, w, codes.ctypes.data_as(C.POINTER(C.c_uint16)), codes.size,
            C.byref(count)))
        return codes[: count.value]

    def features(self, rows_hint=0):
        count = C.c_size_t()
        probe = np.zeros(1, np.float32)
        status = self.lib.lib.omni_context_copy_features(self.handle, probe.ctypes.data_as(C.POINTER(C.c_float)), 0,
                                                         C.byref(count))
        if status not in (0, 1):
            self.lib.check(status)
        out = np.zeros(count.value, np.float32)
        self.lib.check(self.lib.lib.omni_context_copy_features(
            self.handle, out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(count)))
        return out.reshape(rows_hint, -1) if rows_hint else out

    def cancel(self):
        self.lib.lib.omni_context_cancel(self.handle)

    def reset_cancel(self):
        self.lib.lib.omni_context_reset_cancel(self.handle)

    @property
    def peak_workspace(self):
        return int(self.lib.lib.omni_context_peak_workspace(self.handle))

    @property
    def graph_launches(self):
        """CUDA-graph launches of repeated batched calls (captures and replays)."""
        return int(self.lib.lib.omni_b200_context_graph_launches(self.handle))

    def close(self):
        if self.handle:
            self.lib.lib.omni_context_free(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
