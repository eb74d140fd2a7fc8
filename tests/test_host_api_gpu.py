"""Host-buffer entry points (omni_b200_context: the omni_context role of
src/runtime.cpp:200-211): results must equal the device-pointer entry points
bit for bit, for every batch chunking the pipelined copy path uses, and the
context must reject a concurrent call (src/runtime.cpp:152-163)."""

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


@pytest.mark.parametrize("batch,heads,L,D,dtype,varlen", [
    (5, 3, 300, 72, torch.float16, False),   # 5 items -> 5 chunks of one item
    (11, 2, 257, 64, torch.bfloat16, True),  # 11 items -> 8 uneven chunks, key lengths
    (1, 4, 129, 96, torch.bfloat16, False),
])
def test_attention_host_equals_device(ob, batch, heads, L, D, dtype, varlen):
    g = torch.Generator().manual_seed(batch * 131 + L)
    q, k, v = [(torch.randn(batch, heads, L, D, generator=g) * 0.5).to(dtype) for _ in range(3)]
    lengths = torch.randint(1, L + 1, (batch,), generator=g, dtype=torch.int32) if varlen else None
    code = 1 if dtype == torch.bfloat16 else 2
    want = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(),
                             lengths=lengths.cuda() if varlen else None).cpu()
    hq, hk, hv = (t.contiguous().pin_memory() for t in (q, k, v))
    out = torch.empty_like(hq).pin_memory()
    hlen = lengths.numpy() if varlen else None
    with ob.Context(0) as ctx:
        for _ in range(2):  # the second call reuses the context's buffers
            out.zero_()
            ctx.attention_bhld(hq, hk, hv, out, batch, heads, L, D, code, code, lengths=hlen)
            assert torch.equal(out, want)
        assert ctx.peak_workspace_bytes >= 4 * q.numel() * q.element_size()


@pytest.mark.parametrize("profile", [1, 0])
def test_vq_host_equals_oracle(ob, profile):
    rng = np.random.default_rng(5 + profile)
    rows, dim, codes = 1000, 64, 3000
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    cb = rng.standard_normal((codes, dim)).astype(np.float32)
    if profile == 1:
        x, cb = O.round_bf16(x), O.round_bf16(cb)
        hx = torch.from_numpy(x).to(torch.bfloat16)
        hc = torch.from_numpy(cb).to(torch.bfloat16)
    else:
        hx, hc = torch.from_numpy(x), torch.from_numpy(cb)
    ids = np.zeros(rows, np.uint16)
    with ob.Context(0) as ctx:
        ctx.vq_argmin(hx, hc, ids, rows, dim, codes, profile=profile, ids_u16=True)
    want = O.quantize(x, cb, bf16=profile == 1)
    mism = np.nonzero(ids != want)[0]
    if profile == 0:
        assert len(mism) == 0, f"{len(mism)} rows differ"  # fp32 profile: exact
    elif len(mism):
        # bf16 profile: the tie rule, plus rare bf16 rounding-boundary flips of
        # the dot product (same allowance as tests/test_vq_gpu.py).
        d1, d2 = O.quantize_top2(x[mism], cb, bf16=True)
        rest = mism[~((d2 - d1) < 1e-3 * np.abs(d1))]
        assert len(rest) <= max(1, 0.002 * rows), f"{len(rest)} rows differ beyond the tie rule"
