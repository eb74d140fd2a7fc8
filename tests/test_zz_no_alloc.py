"""omni_b200_vq_argmin_noalloc: the VQ argmin for callers that cannot allocate
device memory (their HBM belongs to another allocator, or cudaMalloc/cudaFree
are not allowed in their serving loop).  It must give exactly the ids of
omni_b200_vq_argmin on the same inputs -- it runs the same kernels on a fixed
device scratch array -- on consecutive calls, and reject batches larger than
its fixed scratch.  Collected last so that a failure here cannot hide the
other tests of a `-x` run."""

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_ROWS = 65536


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    lib = load_package().library()
    fn = lib.lib.omni_b200_vq_argmin_noalloc
    P = C.c_void_p
    fn.restype = C.c_int
    fn.argtypes = [P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int, P]
    return lib


def _inputs(rows, dim, codes, seed):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(O.round_bf16(rng.standard_normal((rows, dim)).astype(np.float32))).to(torch.bfloat16).cuda()
    cb = torch.from_numpy(O.round_bf16(rng.standard_normal((codes, dim)).astype(np.float32))).to(torch.bfloat16).cuda()
    return x, cb


def _norms(lib, cb, stream):
    codes, dim = cb.shape
    norms = torch.empty(codes, dtype=torch.bfloat16, device="cuda")
    lib.check(lib.lib.omni_b200_squares(cb.data_ptr(), norms.data_ptr(), codes, dim, 1, 1, stream))
    return norms


def _with_workspace(lib, x, cb, norms, stream):
    rows, dim = x.shape
    codes = cb.shape[0]
    ws_bytes = lib.lib.omni_b200_vq_workspace(rows, dim, codes, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    lib.check(lib.lib.omni_b200_vq_argmin(x.data_ptr(), cb.data_ptr(), norms.data_ptr(), ids.data_ptr(), rows, dim,
                                          codes, 1, 0, ws.data_ptr(), ws_bytes, stream))
    lib.sync_check(stream)
    return ids.cpu()


def _no_alloc(lib, x, cb, norms, stream):
    rows, dim = x.shape
    codes = cb.shape[0]
    ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    lib.check(lib.lib.omni_b200_vq_argmin_noalloc(x.data_ptr(), cb.data_ptr(), norms.data_ptr(), ids.data_ptr(),
                                                  rows, dim, codes, 1, 0, stream))
    lib.sync_check(stream)
    return ids.cpu()


def test_no_alloc_matches_workspace_entry_point_on_consecutive_calls(lib):
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row with different shapes: the second must not see the
    # first call's scratch contents.
    for rows, dim, codes, seed in [(5000, 64, 4099, 1), (777, 32, 16384, 2)]:
        x, cb = _inputs(rows, dim, codes, seed)
        norms = _norms(lib, cb, stream)
        want = _with_workspace(lib, x, cb, norms, stream)
        got = _no_alloc(lib, x, cb, norms, stream)
        assert torch.equal(got, want), f"{int((got != want).sum())} ids differ for rows={rows}"


def test_no_alloc_rejects_batches_beyond_its_scratch(lib):
    stream = torch.cuda.current_stream().cuda_stream
    x, cb = _inputs(8, 64, 300, 3)
    norms = _norms(lib, cb, stream)
    ids = torch.empty(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    st = lib.lib.omni_b200_vq_argmin_noalloc(x.data_ptr(), cb.data_ptr(), norms.data_ptr(), ids.data_ptr(),
                                             MAX_ROWS + 1, 64, 300, 1, 0, stream)
    assert st == 1
    assert b"exceed" in lib.lib.omni_b200_last_error()
    # A successful call after the rejected one leaves no stale message behind.
    ok = torch.empty(8, dtype=torch.int32, device="cuda")
    lib.check(lib.lib.omni_b200_vq_argmin_noalloc(x.data_ptr(), cb.data_ptr(), norms.data_ptr(), ok.data_ptr(),
                                                  8, 64, 300, 1, 0, stream))
    assert lib.lib.omni_b200_last_error() == b""
    lib.sync_check(stream)
