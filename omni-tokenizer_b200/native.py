"""ctypes binding of the op-level C ABI (include/omni_b200.h).

Mirrors the reference's binding style (omni-tokenizer
python/omni_tokenizer/native.py:36-139: one Library object, every signature
declared at load, non-zero status raised as NativeError with the thread-local
message).  No tensor framework is needed here; the helpers at the bottom
accept torch tensors only as holders of device pointers.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent

F32, BF16, F16 = 0, 1, 2

# omni_status (include/omni/omni.h)
OK, INVALID_ARGUMENT, IO_ERROR, INVALID_MODEL, UNSUPPORTED, OUT_OF_MEMORY, CANCELLED, INTERNAL_ERROR = range(8)


class NativeError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


_P = C.c_void_p
SIGNATURES = {
    "omni_b200_last_error": (C.c_char_p, []),
    "omni_b200_version": (C.c_char_p, []),
    "omni_b200_sync_check": (C.c_int, [_P]),
    "omni_b200_wait_selftest": (C.c_int, [C.c_uint, _P]),
    "omni_b200_debug_fail_allocations": (None, [C.c_int]),
    "omni_b200_attention_bhld": (
        C.c_int,
        [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, C.c_float, _P],
    ),
    "omni_b200_attention_rows_workspace": (C.c_size_t, [C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_int]),
    "omni_b200_attention_rows": (
        C.c_int,
        [_P, _P, _P, _P, C.c_size_t, C.c_int, C.c_int, C.c_size_t, C.c_size_t, C.c_int, C.c_int, C.c_int, _P,
         C.c_size_t, _P],
    ),
    "omni_b200_attention_rows_batch_workspace": (
        C.c_size_t, [C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "omni_b200_attention_rows_batch": (
        C.c_int,
        [_P, _P, _P, _P, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_size_t, _P, C.c_int, C.c_int,
         C.c_int, _P, C.c_size_t, _P],
    ),
    "omni_b200_gelu": (C.c_int, [_P, C.c_size_t, C.c_int, _P]),
    "omni_b200_squares": (C.c_int, [_P, _P, C.c_size_t, C.c_size_t, C.c_int, C.c_int, _P]),
    "omni_b200_vq_argmin": (
        C.c_int,
        [_P, _P, _P, _P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int, _P, C.c_size_t, _P],
    ),
    "omni_b200_vq_argmin_cancellable": (
        C.c_int,
        [_P, _P, _P, _P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int, _P, C.c_size_t, _P, _P],
    ),
    "omni_b200_vq_workspace": (C.c_size_t, [C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
    "omni_b200_context_create": (C.c_int, [C.c_int, C.POINTER(_P)]),
    "omni_b200_context_free": (None, [_P]),
    "omni_b200_context_peak_workspace": (C.c_uint64, [_P]),
    "omni_b200_attention_bhld_host": (
        C.c_int,
        [_P, _P, _P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, C.c_float],
    ),
    "omni_b200_vq_argmin_host": (
        C.c_int, [_P, _P, _P, _P, _P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int],
    ),
}


class Library:
    """The B200 hot-path library.  Raises NativeError(UNSUPPORTED) when the
    shared library is missing -- there is no CPU fallback."""

    def __init__(self, path=None):
        explicit = path or os.environ.get("OMNI_B200_LIBRARY")
        found = Path(explicit) if explicit else PKG / "libomni_b200.so"
        if not found.is_file():
            raise NativeError(UNSUPPORTED, f"B200 library not found at {found}; run omni-tokenizer_b200/build.py")
        self.path = found.resolve()
        self.lib = C.CDLL(str(self.path))
        missing = [name for name in SIGNATURES if not hasattr(self.lib, name)]
        if missing:
            raise NativeError(UNSUPPORTED, f"{self.path} lacks {', '.join(missing)}; rebuild it")
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype, fn.argtypes = res, args

    def check(self, status):
        if status:
            msg = self.lib.omni_b200_last_error()
            raise NativeError(status, msg.decode("utf-8", "replace") if msg else f"native error {status}")

    def version(self):
        return self.lib.omni_b200_version().decode()

    def sync_check(self, stream=None):
        self.check(self.lib.omni_b200_sync_check(stream))


_LIB = None


def library() -> Library:
    global _LIB
    if _LIB is None:
        _LIB = Library()
    return _LIB


# ----------------------------------------------------------------- torch helpers
def _dtype_code(t):
    import torch

    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}[t.dtype]


def _stream_ptr(stream):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def attention_bhld(q, k, v, out=None, lengths=None, block=0, skip_padded_queries=False, scale=0.0,
                   out_dtype=None, stream=None):
    """Head-major batched attention: q, k, v are CUDA tensors [B, H, L, D]."""
    import torch

    B, H, L, D = q.shape
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=q.device)
    lib = library()
    lib.check(lib.lib.omni_b200_attention_bhld(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, L, D, _dtype_code(q),
        _dtype_code(out), lengths.data_ptr() if lengths is not None else None, block,
        int(bool(skip_padded_queries)), float(scale), _stream_ptr(stream)))
    return out


class Context:
    """Host-buffer entry points bound to one device (omni_b200_context)."""

    def __init__(self, device=0, lib=None):
        self.lib = lib or library()
        self.handle = C.c_void_p()
        self.lib.check(self.lib.lib.omni_b200_context_create(int(device), C.byref(self.handle)))

    def close(self):
        if self.handle:
            self.lib.lib.omni_b200_context_free(self.handle)
            self.handle = C.c_void_p()

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()

    @property
    def peak_workspace_bytes(self):
        return int(self.lib.lib.omni_b200_context_peak_workspace(self.handle))

    def attention_bhld(self, q, k, v, out, batch, heads, L, head_dim, dtype, out_dtype, lengths=None, block=0,
                       skip_padded_queries=False, scale=0.0):
        """q, k, v, out, lengths: host addresses (ints) or objects with .ctypes.data / .data_ptr()."""
        self.lib.check(self.lib.lib.omni_b200_attention_bhld_host(
            self.handle, _addr(q), _addr(k), _addr(v), _addr(out), batch, heads, L, head_dim, dtype, out_dtype,
            _addr(lengths) if lengths is not None else None, block, int(bool(skip_padded_queries)), float(scale)))

    def vq_argmin(self, x, codebook, ids, rows, dim, codes, profile=BF16, ids_u16=True, cbnorm=None):
        self.lib.check(self.lib.lib.omni_b200_vq_argmin_host(
            self.handle, _addr(x), _addr(codebook), _addr(cbnorm) if cbnorm is not None else None, _addr(ids),
            rows, dim, codes, profile, int(bool(ids_u16))))


def _addr(obj):
    if isinstance(obj, int):
        return obj
    if hasattr(obj, "data_ptr"):
        return obj.data_ptr()
    return obj.ctypes.data


def gelu_(x, stream=None):
    """Ops::gelu in place on a contiguous fp32 or bf16 CUDA tensor."""
    lib = library()
    lib.check(lib.lib.omni_b200_gelu(x.data_ptr(), x.numel(), _dtype_code(x), _stream_ptr(stream)))
    return x


def attention_rows(q, k, v, heads, block=0, valid=None, fused=False, out_dtype=None, stream=None,
                   batch=1, lengths=None, workspace=True):
    """Ops::attention on the reference's row-major layout (CUDA tensors).

    batch > 1: `batch` sequences of q.shape[0] // batch rows each, keys of
    sequence b limited to lengths[b] (a CUDA int32 tensor) when given.
    workspace=False passes only the repacking bytes (no key split scratch)."""
    import torch

    rows = q.shape[0]
    n = rows // batch
    d = q.shape[1] // 3 if fused else q.shape[1]
    hd = d // heads
    valid = n if valid is None else valid
    out = torch.empty((rows, d), dtype=out_dtype or q.dtype, device=q.device)
    lib = library()
    if batch == 1 and lengths is None:
        ws_bytes = lib.lib.omni_b200_attention_rows_workspace(n, heads, hd, _dtype_code(q), int(fused))
    else:
        ws_bytes = lib.lib.omni_b200_attention_rows_batch_workspace(n, batch, heads, hd, _dtype_code(q),
                                                                    int(fused))
    if not workspace:
        ws_bytes = 0
        if _dtype_code(q) == 0 or hd % 8 or (3 * d if fused else d) % 8:
            raise ValueError("workspace=False needs rows that are read in place")
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    if batch == 1 and lengths is None:
        lib.check(lib.lib.omni_b200_attention_rows(
            q.data_ptr(), None if fused else k.data_ptr(), None if fused else v.data_ptr(), out.data_ptr(), n,
            heads, hd, block, valid, int(fused), _dtype_code(q), _dtype_code(out), ws.data_ptr(), ws_bytes,
            _stream_ptr(stream)))
    else:
        lib.check(lib.lib.omni_b200_attention_rows_batch(
            q.data_ptr(), None if fused else k.data_ptr(), None if fused else v.data_ptr(), out.data_ptr(), n,
            batch, heads, hd, block, valid, None if lengths is None else lengths.data_ptr(), int(fused),
            _dtype_code(q), _dtype_code(out), ws.data_ptr(), ws_bytes, _stream_ptr(stream)))
    return out
