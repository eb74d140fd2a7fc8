"""Parity at the BASELINE configurations' full sizes.

The whole batch runs on the GPU exactly as bench.py runs it; the CPU oracle
re-computes a seeded sample of (item, head) slices (attention) or rows (VQ),
which it finishes in seconds, and size-independent properties are checked on
the full output: every value finite, and every attention output row a convex
combination of the value rows it may see (so it lies inside their
per-column range).
"""

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ATTN = {
    # name: (B, H, L, D, dtype, std, seed, varlen)
    "c2": (32, 16, 729, 72, torch.float16, 0.5, 1002, None),
    "c1": (1, 20, 1500, 64, torch.bfloat16, 1.0, 1001, None),
    "c3": (64, 20, 1500, 64, torch.bfloat16, 1.0, 1003, (100, 1500)),
}


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


def _inputs(B, H, L, D, dtype, std, seed, varlen):
    g = torch.Generator().manual_seed(seed)
    q, k, v = [(torch.randn(B, H, L, D, generator=g) * std).to(dtype) for _ in range(3)]
    lengths = None
    if varlen:
        rng = np.random.default_rng(seed)
        lengths = torch.from_numpy(rng.integers(varlen[0], varlen[1] + 1, size=B).astype(np.int32))
    return q, k, v, lengths


@pytest.mark.parametrize("name", ["c2", "c1", "c3"])
def test_attention_full_size(ob, name):
    B, H, L, D, dtype, std, seed, varlen = ATTN[name]
    q, k, v, lengths = _inputs(B, H, L, D, dtype, std, seed, varlen)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    ld = lengths.cuda() if lengths is not None else None
    out = ob.attention_bhld(qd, kd, vd, lengths=ld, skip_padded_queries=varlen is not None)
    torch.cuda.synchronize()
    valid = lengths.cuda().long() if lengths is not None else torch.full((B,), L, device="cuda")

    # Size-independent properties over the whole batch.
    rows = torch.arange(L, device="cuda")
    qmask = (rows[None, :] < valid[:, None])[:, None, :, None]  # [B,1,L,1]
    o = out.float()
    assert torch.isfinite(torch.where(qmask, o, torch.zeros_like(o))).all()
    kmask = qmask  # keys visible to every query: the first `valid` tokens of the item
    vf = vd.float()
    vmax = torch.where(kmask, vf, torch.full_like(vf, -np.inf)).amax(dim=2, keepdim=True)
    vmin = torch.where(kmask, vf, torch.full_like(vf, np.inf)).amin(dim=2, keepdim=True)
    slack = 1e-2 * (vmax - vmin).clamp_min(1e-3)
    inside = (o <= vmax + slack) & (o >= vmin - slack)
    assert torch.where(qmask, inside, torch.ones_like(inside)).all(), "output outside the convex hull of V"

    # Oracle on a seeded sample of (item, head) slices.
    rng = np.random.default_rng(seed + 1)
    picks = [(int(rng.integers(B)), int(rng.integers(H))) for _ in range(3 if name != "c2" else 5)]
    for b, h in picks:
        n = int(valid[b])
        qs = q[b:b + 1, h:h + 1].float().numpy()
        ks = k[b:b + 1, h:h + 1].float().numpy()
        vs = v[b:b + 1, h:h + 1].float().numpy()
        want = O.attention_bhld(qs, ks, vs, lengths=np.array([n], np.int32))[0, 0, :n]
        got = out[b, h, :n].float().cpu().numpy()
        err = np.abs(got - want)
        assert err.max() <= 2e-2 and err.mean() <= 2e-3, (name, b, h, float(err.max()), float(err.mean()))


@pytest.mark.parametrize("name,N,K,dim,seed,sample", [("vq_audio", 24000, 16384, 64, 1010, 600),
                                                      ("vq_image", 373248, 16384, 32, 1011, 400)])
def test_vq_full_size(ob, name, N, K, dim, seed, sample):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, dim, generator=g).to(torch.bfloat16)
    cb = torch.randn(K, dim, generator=g).to(torch.bfloat16)
    xd, cd = x.cuda(), cb.cuda()
    lib = ob.library()
    stream = torch.cuda.current_stream().cuda_stream
    norms = torch.empty(K, dtype=torch.bfloat16, device="cuda")
    lib.check(lib.lib.omni_b200_squares(cd.data_ptr(), norms.data_ptr(), K, dim, 1, 1, stream))
    ws_bytes = lib.lib.omni_b200_vq_workspace(N, dim, K, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    lib.check(lib.lib.omni_b200_vq_argmin(xd.data_ptr(), cd.data_ptr(), norms.data_ptr(), ids.data_ptr(), N, dim,
                                          K, 1, 0, ws.data_ptr(), ws_bytes, stream))
    lib.sync_check()
    got = ids.cpu().numpy()
    assert got.min() >= 0 and got.max() < K
    rows = np.sort(np.random.default_rng(seed + 1).choice(N, size=sample, replace=False))
    xs = x[rows].float().numpy()
    cbf = cb.float().numpy()
    from tests.test_vq_gpu import _check

    _check(xs, cbf, got[rows].astype(np.int64), what=f"{name} sample of {sample} rows")
