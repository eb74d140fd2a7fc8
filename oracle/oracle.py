"""ctypes access to the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs import this module.  It is the checker for the CUDA kernels,
never the thing measured or shipped: the product library
(omni-tokenizer_b200/) does not import it.

Two libraries:
  * oracle/liboracle.so        -- oracle/omni_oracle.c, a C restatement of the
                                  reference's src/cpu.cpp arithmetic (always
                                  buildable with gcc from this repository);
  * oracle/_ref/libomni_ref_cpu.so -- the reference's own src/cpu.cpp compiled
                                  unchanged (oracle/Makefile `ref`); present only
                                  where the reference checkout was available at
                                  build time.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_F = C.POINTER(C.c_float)
_D = C.POINTER(C.c_double)
_U16 = C.POINTER(C.c_uint16)
_I32 = C.POINTER(C.c_int32)
_SZ = C.c_size_t

_lib = None
_ref = None


def _build(target=None):
    cmd = ["make", "-s", "-C", str(HERE)] + ([target] if target else [])
    subprocess.run(cmd, check=True, capture_output=True)


def lib():
    """The C restatement (built on first use if the .so is missing)."""
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.is_file() or path.stat().st_mtime < (HERE / "omni_oracle.c").stat().st_mtime:
            _build()
        L = C.CDLL(str(path))
        L.oracle_round_bf16.restype = C.c_float
        L.oracle_round_bf16.argtypes = [C.c_float]
        L.oracle_attention.restype = None
        L.oracle_attention.argtypes = [_F, _F, _F, _F, _SZ, _SZ, _SZ, _SZ, _SZ, C.c_int, C.c_int]
        L.oracle_attention_bhld.restype = None
        L.oracle_attention_bhld.argtypes = [_F, _F, _F, _F, _SZ, _SZ, _SZ, _SZ, _I32, _SZ]
        L.oracle_squares.restype = None
        L.oracle_squares.argtypes = [_F, _F, _SZ, _SZ, C.c_int]
        L.oracle_quantize.restype = None
        L.oracle_quantize.argtypes = [_F, _SZ, _SZ, _F, _SZ, _F, C.c_int, _U16, _D]
        L.oracle_quantize_top2.restype = None
        L.oracle_quantize_top2.argtypes = [_F, _SZ, _SZ, _F, _SZ, _F, C.c_int, _D, _D]
        L.oracle_lcg_values.restype = None
        L.oracle_lcg_values.argtypes = [_F, _SZ, C.c_uint32]
        L.oracle_fp32_distance_error_factor.restype = C.c_double
        L.oracle_fp32_distance_error_factor.argtypes = [_SZ]
        _lib = L
    return _lib


def ref_available():
    return (HERE / "_ref" / "libomni_ref_cpu.so").is_file()


def ref():
    """The reference's own cpu.cpp (None when it was not built here)."""
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libomni_ref_cpu.so"
        if not path.is_file():
            return None
        L = C.CDLL(str(path))
        L.ref_attention.restype = C.c_int
        L.ref_attention.argtypes = [_F, _F, _F, _F, _SZ, _SZ, _SZ, _SZ, _SZ, C.c_int, C.c_int]
        L.ref_squares.restype = C.c_int
        L.ref_squares.argtypes = [_F, _F, _SZ, _SZ, C.c_int]
        L.ref_quantize.restype = C.c_int
        L.ref_quantize.argtypes = [_F, _SZ, _SZ, _F, _SZ, _F, C.c_int, _U16]
        _ref = L
    return _ref


def _f(a):
    return a.ctypes.data_as(_F)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def round_bf16(x):
    """Vectorised omni-tokenizer src/internal.h:128-139 (RNE, NaN quieted)."""
    x = f32(x)
    u = x.view(np.uint32).copy()
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    u = np.where(
        nan,
        u | np.uint32(0x00400000),
        u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)),
    ).astype(np.uint32)
    return (u & np.uint32(0xFFFF0000)).view(np.float32)


def lcg_values(count, seed):
    """The generator of the reference's native tests (values in [-1, 1))."""
    out = np.empty(count, np.float32)
    lib().oracle_lcg_values(_f(out), count, seed)
    return out


def attention(q, k, v, heads, block=0, valid=None, fused=False, bf16=False, impl="oracle"):
    """Ops::attention on [n, cols] row-major inputs; returns [n, d] float32.

    impl="oracle" runs the C restatement, impl="ref" the reference's cpu.cpp.
    Inputs are rounded to bf16 first when bf16=True (as Ops::upload does).
    """
    q = f32(q)
    n, cols = q.shape
    d = cols // 3 if fused else cols
    valid = n if valid is None else valid
    if bf16 and impl == "oracle":
        q = round_bf16(q)
    if fused:
        k = v = np.zeros((1, 1), np.float32)
    else:
        k, v = f32(k), f32(v)
        if bf16 and impl == "oracle":
            k, v = round_bf16(k), round_bf16(v)
    y = np.zeros((n, d), np.float32)
    if impl == "ref":
        status = ref().ref_attention(_f(q), _f(k), _f(v), _f(y), n, cols, heads, block, valid, int(fused), int(bf16))
        assert status == 0
    else:
        lib().oracle_attention(_f(q), _f(k), _f(v), _f(y), n, cols, heads, block, valid, int(fused), int(bf16))
    return y


def attention_bhld(q, k, v, lengths=None, block=0):
    """Head-major batched attention [B, H, L, D] with optional per-item key lengths."""
    q, k, v = f32(q), f32(k), f32(v)
    B, H, L, D = q.shape
    y = np.zeros_like(q)
    lens = None
    if lengths is not None:
        lens = np.ascontiguousarray(lengths, dtype=np.int32)
    lib().oracle_attention_bhld(
        _f(q), _f(k), _f(v), _f(y), B, H, L, D,
        lens.ctypes.data_as(_I32) if lens is not None else None, block,
    )
    return y


def squares(x, bf16=False, impl="oracle"):
    x = f32(x)
    rows, cols = x.shape
    if bf16 and impl == "oracle":
        x = round_bf16(x)
    y = np.zeros(rows, np.float32)
    if impl == "ref":
        assert ref().ref_squares(_f(x), _f(y), rows, cols, int(bf16)) == 0
    else:
        lib().oracle_squares(_f(x), _f(y), rows, cols, int(bf16))
    return y


def quantize(x, codebook, cbnorm=None, bf16=False, impl="oracle", return_best=False):
    """Ops::quantize: nearest codebook row ids (uint16) per row of x."""
    x, cb = f32(x), f32(codebook)
    if bf16 and impl == "oracle":
        x, cb = round_bf16(x), round_bf16(cb)
    if cbnorm is None:
        cbnorm = squares(cb, bf16=bf16)
    cbnorm = f32(cbnorm)
    if bf16 and impl == "oracle":
        cbnorm = round_bf16(cbnorm)
    rows, dim = x.shape
    codes = cb.shape[0]
    ids = np.zeros(rows, np.uint16)
    best = np.zeros(rows, np.float64)
    if impl == "ref":
        assert ref().ref_quantize(_f(x), rows, dim, _f(cb), codes, _f(cbnorm), int(bf16), ids.ctypes.data_as(_U16)) == 0
    else:
        lib().oracle_quantize(
            _f(x), rows, dim, _f(cb), codes, _f(cbnorm), int(bf16),
            ids.ctypes.data_as(_U16), best.ctypes.data_as(_D),
        )
    return (ids, best) if return_best else ids


def quantize_top2(x, codebook, cbnorm=None, bf16=False):
    x, cb = f32(x), f32(codebook)
    if bf16:
        x, cb = round_bf16(x), round_bf16(cb)
    if cbnorm is None:
        cbnorm = squares(cb, bf16=bf16)
    cbnorm = f32(cbnorm)
    if bf16:
        cbnorm = round_bf16(cbnorm)
    rows, dim = x.shape
    d1 = np.zeros(rows, np.float64)
    d2 = np.zeros(rows, np.float64)
    lib().oracle_quantize_top2(
        _f(x), rows, dim, _f(cb), cb.shape[0], _f(cbnorm), int(bf16),
        d1.ctypes.data_as(_D), d2.ctypes.data_as(_D),
    )
    return d1, d2


def cpu_threads():
    """Threads OpenMP will use in this process (OMP_NUM_THREADS or all cores)."""
    env = os.environ.get("OMP_NUM_THREADS")
    return int(env) if env else (len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count())
