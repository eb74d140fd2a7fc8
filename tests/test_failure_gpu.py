"""Failure detection, exercised without faulting or hanging a GPU.

* Bounded waits: every pipeline wait in the kernels gives up after a limit,
  records a bit in the device's kernel error word and lets the kernel end.
  omni_b200_wait_selftest runs that same wait on a barrier that nothing
  completes, with a limit of a few milliseconds; omni_b200_sync_check must then
  report OMNI_INTERNAL_ERROR, and the device must stay usable.
* Out of memory: omni_b200_debug_fail_allocations makes the library's next
  device allocations fail on the host side (no allocator call).  The status is
  OMNI_OUT_OF_MEMORY, as the reference maps CUDA allocation failures
  (src/cuda.cu:18-22); the encoder contexts trim their memory pool and retry
  once, as the reference's Pool does (src/cuda.cu:515-527).
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "encoder"
INTERNAL_ERROR, OUT_OF_MEMORY = 7, 5


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


@pytest.fixture()
def hook(ob):
    lib = ob.library().lib
    yield lib.omni_b200_debug_fail_allocations
    lib.omni_b200_debug_fail_allocations(0)


def _small_attention_ok(ob):
    g = torch.Generator().manual_seed(5)
    q, k, v = [torch.randn(1, 2, 130, 64, generator=g).to(torch.bfloat16) for _ in range(3)]
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), out_dtype=torch.float32)
    ob.library().sync_check()
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy())
    assert np.abs(out.cpu().numpy() - want).max() <= 2e-2


def test_bounded_wait_gives_up_and_is_reported(ob):
    lib = ob.library()
    stream = torch.cuda.current_stream().cuda_stream
    lib.sync_check(stream)  # start from a clear error word
    assert lib.lib.omni_b200_wait_selftest(0, stream) == 1
    assert lib.lib.omni_b200_wait_selftest(3_000_000, stream) == 1
    assert lib.lib.omni_b200_wait_selftest(5000, stream) == 0  # 5 ms
    assert lib.lib.omni_b200_sync_check(stream) == INTERNAL_ERROR
    msg = lib.lib.omni_b200_last_error()
    assert b"timed out" in msg and b"200" in msg, msg
    # The check cleared the word, and the device still computes correctly.
    assert lib.lib.omni_b200_sync_check(stream) == 0
    _small_attention_ok(ob)


def test_forced_allocation_failure_in_host_context(ob, hook):
    g = torch.Generator().manual_seed(6)
    q, k, v = [torch.randn(2, 2, 100, 64, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3)]
    out = torch.empty_like(q).pin_memory()
    with ob.Context(0) as ctx:
        hook(1)
        with pytest.raises(ob.NativeError) as e:
            ctx.attention_bhld(q, k, v, out, 2, 2, 100, 64, 1, 1)
        assert e.value.status == OUT_OF_MEMORY and "device buffer" in str(e.value)
        # The hook is used up; the same context works.
        ctx.attention_bhld(q, k, v, out, 2, 2, 100, 64, 1, 1)
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy())
    assert np.abs(out.float().numpy() - want).max() <= 2e-2


def test_forced_allocation_failure_in_encoder(ob, hook):
    import omni_tokenizer_b200.abi as abi

    golden = dict(np.load(GOLDEN / "golden.npz"))
    ours = abi.OmniLib(ob.library().path)
    px = golden["image0_pixels"]
    # A weight allocation that fails makes the load fail with OUT_OF_MEMORY.
    hook(1)
    with pytest.raises(abi.OmniError) as e:
        ours.load(GOLDEN / "image.omni")
    assert e.value.status == OUT_OF_MEMORY
    hook(0)
    with ours.load(GOLDEN / "image.omni") as m:
        s = m.context()
        want = s.encode_image(px)
        # One failed activation allocation: the pool is trimmed and the retry succeeds.
        hook(1)
        assert np.array_equal(s.encode_image(px), want)
        # Two in a row: OUT_OF_MEMORY, with the reference's message shape.
        hook(2)
        with pytest.raises(abi.OmniError) as e:
            s.encode_image(px)
        assert e.value.status == OUT_OF_MEMORY and "allocation" in str(e.value)
        hook(0)
        # The context is still usable and gives the same codes.
        assert np.array_equal(s.encode_image(px), want)
        s.close()


def test_cancel_reaches_the_vq_pass(ob):
    """Cancellation between the last layer and the codes: the reference's next
    check after its layer loop is in Ops::quantize, before every codebook tile
    (src/cuda.cu:946-948).  Here a trace callback cancels at the last layer; the
    VQ launches read the context's flag when they start and skip their codebook
    windows, and the call reports OMNI_CANCELLED.  After a reset the context
    gives the uncancelled codes again."""
    import omni_tokenizer_b200.abi as abi

    golden = dict(np.load(GOLDEN / "golden.npz"))
    ours = abi.OmniLib(ob.library().path)
    lib = ours.lib
    mel, valid = golden["audio1_mel"], int(golden["audio1_valid"])
    with ours.load(GOLDEN / "audio.omni") as m:
        s = m.context()
        want = s.encode_audio(mel, valid)
        layers = m.info().layers
        seen = []

        def cb(user, stage, values, rows, cols):
            seen.append(stage.decode())
            if stage.decode() == f"layer.{layers - 1}":
                lib.omni_context_cancel(s.handle)

        fn = abi.TRACE(cb)
        assert lib.omni_context_set_trace(s.handle, fn, None) == 0
        with pytest.raises(abi.OmniError) as e:
            s.encode_audio(mel, valid)
        assert e.value.status == 6
        assert seen[-1] == f"layer.{layers - 1}"  # no stage after the last layer ran on the host
        assert lib.omni_context_set_trace(s.handle, abi.TRACE(0), None) == 0
        s.reset_cancel()
        assert np.array_equal(s.encode_audio(mel, valid), want)
        s.close()
