"""GPU parity of the sm_100a attention kernel against the CPU oracle.

Tolerance: for bf16/fp16 inputs, max-abs error <= 2e-2
and mean-abs error <= 2e-3 against the reference's fp32 CPU attention
(src/cpu.cpp:122-172) run on the same (bf16/fp16-representable) values.
Every test calls the CUDA kernel through the C ABI (include/omni_b200.h).
"""

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


def _close(got, want, what=""):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err.max() <= MAX_ABS, f"{what}: max-abs {err.max():.3e}"
    assert err.mean() <= MEAN_ABS, f"{what}: mean-abs {err.mean():.3e}"
    return err.max(), err.mean()


def _bhld_inputs(B, H, L, D, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    qkv = [(torch.randn(B, H, L, D, generator=g) * scale).to(dtype) for _ in range(3)]
    return qkv


@pytest.mark.parametrize(
    "B,H,L,D,dtype",
    [
        (1, 2, 300, 64, torch.bfloat16),   # Whisper-shaped head dim, partial tiles
        (2, 2, 729, 72, torch.float16),    # SigLIP-shaped head dim (72 -> 80 in the tile)
        (1, 3, 257, 96, torch.bfloat16),   # production image head dim
        (1, 1, 1, 64, torch.bfloat16),     # single token
        (1, 2, 1500, 64, torch.bfloat16),  # config 1 length
        (1, 2, 130, 128, torch.float16),
        (2, 1, 200, 32, torch.bfloat16),
        (1, 2, 77, 16, torch.float16),
    ],
)
def test_bhld_matches_oracle(ob, B, H, L, D, dtype):
    q, k, v = _bhld_inputs(B, H, L, D, dtype, seed=B * 1000 + L + D, scale=0.5 if dtype == torch.float16 else 1.0)
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), out_dtype=torch.float32)
    ob.library().sync_check()
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy())
    _close(out.cpu().numpy(), want, f"B{B} H{H} L{L} D{D}")


def test_bhld_key_padding_lengths(ob):
    """Config-3 style varlen batch: padded keys are masked, padded queries ignored."""
    B, H, L, D = 4, 2, 700, 64
    q, k, v = _bhld_inputs(B, H, L, D, torch.bfloat16, seed=7)
    lengths = torch.tensor([100, 333, 700, 513], dtype=torch.int32)
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), lengths=lengths.cuda(), skip_padded_queries=True,
                            out_dtype=torch.float32)
    ob.library().sync_check()
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy(), lengths=lengths.numpy())
    got = out.cpu().numpy()
    for b, n in enumerate(lengths.tolist()):
        _close(got[b, :, :n], want[b, :, :n], f"segment {b} (valid {n})")


@pytest.mark.parametrize("skip", [False, True])
def test_bhld_ragged_lengths_sorted_order(ob, skip):
    """Variable lengths (empty, one key, ragged, full) take the longest-first
    item order across the persistent CTAs: every item is computed exactly once,
    rows of empty sequences are zeros (when computed), padded query rows are
    left untouched when skipped."""
    B, H, L, D = 23, 3, 900, 64
    q, k, v = _bhld_inputs(B, H, L, D, torch.bfloat16, seed=29)
    rng = np.random.default_rng(29)
    lens = rng.integers(1, L + 1, size=B)
    lens[[0, 5]] = 0
    lens[[1, 9]] = 1
    lens[[2, 17]] = L
    lengths = torch.tensor(lens, dtype=torch.int32)
    out = torch.full((B, H, L, D), 7.0, dtype=torch.float32, device="cuda")
    ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), out=out, lengths=lengths.cuda(), skip_padded_queries=skip)
    ob.library().sync_check()
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy(), lengths=lens)
    got = out.cpu().numpy()
    for b, n in enumerate(lens.tolist()):
        if n == 0:
            rows = got[b, :, : (0 if skip else L)]
            assert np.all(rows == 0.0), f"segment {b}: an empty sequence gives zeros"
        else:
            _close(got[b, :, :n], want[b, :, :n], f"segment {b} (valid {n})")
        if skip:
            first_untouched = -(-n // 256) * 256  # whole 256-row items past the length are skipped
            assert np.all(got[b, :, first_untouched:] == 7.0), f"segment {b}: skipped rows written"


def test_bhld_block_causal(ob):
    B, H, L, D = 1, 2, 601, 64
    q, k, v = _bhld_inputs(B, H, L, D, torch.bfloat16, seed=11)
    lengths = torch.tensor([590], dtype=torch.int32)
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), lengths=lengths.cuda(), block=200,
                            out_dtype=torch.float32)
    ob.library().sync_check()
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy(), lengths=lengths.numpy(),
                            block=200)
    _close(out.cpu().numpy(), want, "block 200")


def test_bhld_bf16_output_dtype(ob):
    q, k, v = _bhld_inputs(2, 4, 500, 64, torch.bfloat16, seed=5)
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda())
    ob.library().sync_check()
    assert out.dtype == torch.bfloat16
    want = O.attention_bhld(q.float().numpy(), k.float().numpy(), v.float().numpy())
    _close(out.float().cpu().numpy(), want, "bf16 out")


# Ops::attention on the reference's row-major layout (shapes of
# tests/native_cuda_attention.cpp:233-245 and tests/native_cpu_attention.cpp:129-134).
ROW_CASES = [
    # n, heads, hd, block, valid, fused, dtype
    (1, 2, 7, 0, 1, False, torch.float32),
    (129, 2, 7, 0, 129, False, torch.float32),
    (513, 4, 64, 200, 510, False, torch.float32),
    (1500, 4, 64, 200, 1497, False, torch.float32),
    (401, 2, 7, 7, 1, False, torch.float32),
    (17, 3, 7, 5, 11, True, torch.bfloat16),
    (257, 3, 17, 200, 205, False, torch.float32),
    (31, 2, 96, 0, 31, True, torch.bfloat16),
    (576, 16, 96, 0, 576, True, torch.bfloat16),
    (2049, 2, 96, 0, 2049, True, torch.bfloat16),
    (300, 2, 64, 0, 300, False, torch.bfloat16),
    (150, 2, 72, 0, 150, False, torch.bfloat16),
]


@pytest.mark.parametrize("n,heads,hd,block,valid,fused,dtype", ROW_CASES)
def test_rows_matches_oracle(ob, n, heads, hd, block, valid, fused, dtype):
    d = heads * hd
    cols = 3 * d if fused else d
    q = O.lcg_values(n * cols, 123).reshape(n, cols)
    k = O.lcg_values(n * d, 456).reshape(n, d)
    v = O.lcg_values(n * d, 789).reshape(n, d)
    bf16 = dtype == torch.bfloat16
    tq = torch.from_numpy(q).to(dtype).cuda()
    tk = torch.from_numpy(k).to(dtype).cuda()
    tv = torch.from_numpy(v).to(dtype).cuda()
    out = ob.attention_rows(tq, tk, tv, heads, block=block, valid=valid, fused=fused, out_dtype=torch.float32)
    ob.library().sync_check()
    # The oracle sees the same values the GPU saw (bf16-rounded when bf16), fp32 output.
    want = O.attention(O.round_bf16(q) if bf16 else q, O.round_bf16(k) if bf16 else k,
                       O.round_bf16(v) if bf16 else v, heads, block, valid, fused, bf16=False)
    _close(out.cpu().numpy(), want, f"rows n{n} h{heads} hd{hd} block{block} valid{valid}")


# Key split of a partial last round (16-bit operands): the (query block, head)
# items of a last round that would leave most SMs idle are cut along the keys
# into parts on the idle SMs and merged by a second pass.  The split runs when
# the workspace holds its scratch (the workspace query sizes it);
# workspace=False runs the same call unsplit.
SPLIT_ROW_CASES = [
    # n, heads, hd, block, valid, fused
    (1200, 4, 72, 0, 1200, False),    # 20 items: 7 parts of 1-2 of 10 KV tiles (head dim 72 -> 80)
    (2049, 2, 96, 0, 2049, True),     # 18 items: 8 parts of 2-3 of 17 tiles
    (1000, 4, 64, 0, 900, False),     # 16 items, keys limited to 900: 8 parts of one of the 8 tiles
    (1500, 2, 64, 0, 1500, True),     # 12 items: 8 parts of 1-2 of 12 tiles
    (1024, 2, 128, 0, 1024, False),   # 8 items: 8 parts of one tile
    (1500, 3, 32, 0, 1450, True),     # 18 items, head dim 32
    (1500, 2, 64, 200, 1497, True),   # block window: parts past a row's window, empty parts
    (1000, 4, 64, 300, 1000, False),
    (1500, 2, 64, 1500, 1500, False), # a window as long as the sequence limits nothing
]


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,heads,hd,block,valid,fused", SPLIT_ROW_CASES)
def test_rows_key_split_matches_oracle(ob, n, heads, hd, block, valid, fused, out_dtype):
    lib = ob.library()
    assert lib.lib.omni_b200_attention_rows_workspace(n, heads, hd, 1, int(fused)) > 0  # a split is planned
    d = heads * hd
    cols = 3 * d if fused else d
    q = O.round_bf16(O.lcg_values(n * cols, 321).reshape(n, cols))
    k = O.round_bf16(O.lcg_values(n * d, 654).reshape(n, d))
    v = O.round_bf16(O.lcg_values(n * d, 987).reshape(n, d))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    kw = dict(block=block, valid=valid, fused=fused, out_dtype=out_dtype)
    split = ob.attention_rows(tq, tk, tv, heads, **kw)
    plain = ob.attention_rows(tq, tk, tv, heads, workspace=False, **kw)
    lib.sync_check()
    want = O.attention(q, k, v, heads, block, valid, fused, bf16=False)
    got = split.float().cpu().numpy()
    what = f"n{n} h{heads} hd{hd} block{block} valid{valid}"
    _close(got, want, "split " + what)
    _close(plain.float().cpu().numpy(), want, "unsplit " + what)
    # The parts round P relative to their own row maxima: the two runs agree to
    # within the rounding of P, not bit for bit.
    assert np.abs(got - plain.float().cpu().numpy()).max() <= 1e-2


@pytest.mark.parametrize("heads,lens,block", [
    (16, [1500, 1100], 0),     # 192 items: 148 whole, the 44 of the shorter sequence in 3 parts
    (16, [1500, 1100], 1500),  # the audio graphs' window of the whole sequence: the same plan
    (16, [1500, 90], 0),       # the short sequence's items have one KV tile: two empty parts each
    (16, [1500, 0], 0),        # an empty sequence: every part empty, rows of zeros
    (8, [1000], 0),            # one sequence with a device length: 48 items in 3 parts
    (8, [1000], 256),          # ... with a block window
])
def test_rows_batch_key_split_with_lengths(ob, heads, lens, block):
    """Stacked sequences with device key lengths, as the encoder's batched audio
    call runs them: items in longest-first order, the last round's items split
    along the keys (parts past a short sequence's tiles are empty)."""
    n, hd, batch = 1500, 64, len(lens)
    d = heads * hd
    lib = ob.library()
    assert lib.lib.omni_b200_attention_rows_batch_workspace(n, batch, heads, hd, 1, 1) > 0
    q = O.round_bf16(O.lcg_values(batch * n * 3 * d, 77).reshape(batch * n, 3 * d))
    tq = torch.from_numpy(q).to(torch.bfloat16).cuda()
    lengths = torch.tensor(lens, dtype=torch.int32).cuda()
    out = ob.attention_rows(tq, None, None, heads, block=block, fused=True, batch=batch, lengths=lengths,
                            out_dtype=torch.float32)
    out16 = ob.attention_rows(tq, None, None, heads, block=block, fused=True, batch=batch, lengths=lengths)
    lib.sync_check()
    got, got16 = out.cpu().numpy(), out16.float().cpu().numpy()
    for b, m in enumerate(lens):
        rows = slice(b * n, (b + 1) * n)
        if m == 0:
            assert np.all(got[rows] == 0.0) and np.all(got16[rows] == 0.0), f"sequence {b}: zeros"
            continue
        want = O.attention(q[rows], None, None, heads, block, m, True, bf16=False)
        _close(got[rows], want, f"sequence {b} (valid {m})")
        _close(got16[rows], want, f"sequence {b} (valid {m}, bf16 out)")


@pytest.mark.parametrize("n,hd", [(401, 64), (601, 7), (1025, 64)])
def test_mask_semantics(ob, n, hd):
    """tests/native_cuda_attention.cpp:199-218 through the rows entry point."""
    heads, block, valid = 2, 200, 205
    d = heads * hd
    zero = torch.zeros(n, d, dtype=torch.float32)
    v = torch.tensor([[t + j + 1 for j in range(d)] for t in range(n)], dtype=torch.float32)

    def run(vv):
        out = ob.attention_rows(zero.cuda(), zero.cuda(), vv.cuda(), heads, block=block, valid=valid)
        ob.library().sync_check()
        return out.cpu()

    before = run(v)
    v2 = v.clone()
    v2[valid:] = 10000.0
    invalid_changed = run(v2)
    assert torch.equal(before, invalid_changed), "invalid keys affected attention"
    v2[block:valid] = -10000.0
    future_changed = run(v2)
    assert torch.equal(before[:block], future_changed[:block]), "a future block affected earlier queries"
    assert before[-1, -1] != 0 and before[-1, -1] != future_changed[-1, -1], "padded queries lost access"


def test_invalid_arguments_fail_loudly(ob):
    lib = ob.library()
    q = torch.zeros(1, 1, 8, 60, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ob.NativeError) as e:
        ob.attention_bhld(q, q, q)  # head_dim 60 is not a multiple of 8
    assert e.value.status == 4
    st = lib.lib.omni_b200_attention_bhld(None, None, None, None, 1, 1, 1, 64, 1, 1, None, 0, 0, 0.0, None)
    assert st == 1 and b"null" in lib.lib.omni_b200_last_error()


# ---------------------------------------------------------------------------
# The reference's own CUDA gate (tests/native_cuda_attention.cpp:43-95): inputs
# from its LCG (fused Q|K|V rounded to bf16), output in the input's type, and
# every element of the boundary query rows within a fixed bound of a float64
# scalar attention computed from the same values -- 2e-3 for the fused bf16
# path, 3e-6 for unfused fp32.
def reference_boundary_rows(n, block, valid):
    """Query rows the reference checks: the ends, the valid tail and both
    sides of the 128 / 256 / block / valid boundaries."""
    rows = {0, n - 1, min(n - 1, valid - 1)}
    for boundary in (128, 256, block, valid):
        if boundary and boundary <= n:
            rows.add(boundary - 1)
        if boundary < n:
            rows.add(boundary)
    return sorted(rows)


def reference_rows_fp64(q, k, v, n, heads, hd, block, valid, fused, rows):
    """native_cuda_attention.cpp:62-90 restated: scores as float64 sums of
    float32 products (Q, and for fused inputs also K, pre-multiplied by the
    float32 scale), softmax and the weighted values in float64."""
    d = heads * hd
    f32 = np.float32
    scale = f32(float(hd) ** -0.25) if fused else f32(1) / np.sqrt(f32(hd))
    out = np.zeros((len(rows), d), np.float64)
    for i, t in enumerate(rows):
        limit = min(n, valid)
        if block:
            limit = min(limit, (t // block + 1) * block)
        for h in range(heads):
            a = (q[t, h * hd:(h + 1) * hd] * scale).astype(np.float64)
            if fused:
                kk = (q[:limit, d + h * hd:d + (h + 1) * hd] * scale).astype(np.float64)
                vv = q[:limit, 2 * d + h * hd:2 * d + (h + 1) * hd].astype(np.float64)
            else:
                kk = k[:limit, h * hd:(h + 1) * hd].astype(np.float64)
                vv = v[:limit, h * hd:(h + 1) * hd].astype(np.float64)
            s = kk @ a
            p = np.exp(s - s.max())
            out[i, h * hd:(h + 1) * hd] = (p / p.sum()) @ vv
    return out


FUSED_BF16_CASES = [(n, 2) for n in (31, 32, 129, 255, 256, 257, 385, 512, 2049)] + \
                   [(n, 16) for n in (1, 129, 257, 576, 768, 1080, 2049)]


@pytest.mark.parametrize("n,heads", FUSED_BF16_CASES)
def test_reference_fused_bf16_per_element(ob, n, heads):
    """native_cuda_attention.cpp:238-241: fused hd 96, bf16, bound 2e-3 per element."""
    hd, block, valid = 96, 0, n
    d = heads * hd
    q = O.round_bf16(O.lcg_values(n * 3 * d, 123).reshape(n, 3 * d))
    tq = torch.from_numpy(q).to(torch.bfloat16).cuda()
    out = ob.attention_rows(tq, None, None, heads, block=block, valid=valid, fused=True)
    ob.library().sync_check()
    assert out.dtype == torch.bfloat16
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    rows = reference_boundary_rows(n, block, valid)
    want = reference_rows_fp64(q, None, None, n, heads, hd, block, valid, True, rows)
    err = np.abs(got[rows].astype(np.float64) - want)
    assert err.max() <= 2e-3, f"n={n} heads={heads}: max error {err.max():.3e} at rows {rows}"


# native_cuda_attention.cpp:233-242: the unfused fp32 list, bound 3e-6 per element.
FP32_CASES = []
for _n in (1, 129, 257, 511, 512, 513, 1500, 201, 401):
    FP32_CASES += [(_n, 2, 7, 0, _n), (_n, 4, 64, 200, _n - 3 if _n > 3 else 1), (_n, 2, 7, 7, 1)]
FP32_CASES.append((1, 4, 64, 200, 5))
FP32_BOUND = 3e-6


@pytest.mark.parametrize("n,heads,hd,block,valid", FP32_CASES)
def test_reference_fp32_per_element(ob, n, heads, hd, block, valid):
    """fp32 inputs run the split-precision (3 x tf32) kernel with no 16-bit
    conversion; every element of the reference's boundary rows is within
    3e-6 of the float64 attention of the same values."""
    d = heads * hd
    q = O.lcg_values(n * d, 123).reshape(n, d)
    k = O.lcg_values(n * d, 456).reshape(n, d)
    v = O.lcg_values(n * d, 789).reshape(n, d)
    out = ob.attention_rows(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                            heads, block=block, valid=valid, out_dtype=torch.float32)
    ob.library().sync_check()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    rows = reference_boundary_rows(n, block, valid)
    want = reference_rows_fp64(q, k, v, n, heads, hd, block, valid, False, rows)
    err = np.abs(got[rows].astype(np.float64) - want)
    assert err.max() <= FP32_BOUND, f"n={n} heads={heads} hd={hd} block={block} valid={valid}: {err.max():.3e}"


def _bhld_fp64(q, k, v, b, h, t, limit):
    scale = np.float32(1) / np.sqrt(np.float32(q.shape[-1]))
    a = (q[b, h, t] * scale).astype(np.float64)
    s = k[b, h, :limit].astype(np.float64) @ a
    p = np.exp(s - s.max())
    return (p / p.sum()) @ v[b, h, :limit].astype(np.float64)


@pytest.mark.parametrize("B,H,L,D,lengths,block", [
    (3, 2, 700, 64, (100, 333, 700), 0),     # key padding (BASELINE config 3 semantics)
    (2, 3, 1500, 64, (1500, 1203), 200),     # production audio: block-causal + valid prefix
    (1, 2, 300, 128, None, 0),               # wide heads (32-key tiles)
    (2, 2, 257, 32, (257, 5), 0),
])
def test_bhld_fp32_per_element(ob, B, H, L, D, lengths, block):
    g = torch.Generator().manual_seed(L + D)
    q, k, v = [torch.rand(B, H, L, D, generator=g) * 2 - 1 for _ in range(3)]
    lt = torch.tensor(lengths, dtype=torch.int32).cuda() if lengths else None
    out = ob.attention_bhld(q.cuda(), k.cuda(), v.cuda(), lengths=lt, block=block, out_dtype=torch.float32)
    ob.library().sync_check()
    got = out.cpu().numpy()
    qn, kn, vn = q.numpy(), k.numpy(), v.numpy()
    rng = np.random.default_rng(B * L)
    worst = 0.0
    for b in range(B):
        valid = lengths[b] if lengths else L
        for t in sorted({0, L - 1, valid - 1, *rng.integers(0, L, size=6).tolist()}):
            limit = min(L, valid, (t // block + 1) * block if block else L)
            for h in range(H):
                want = _bhld_fp64(qn, kn, vn, b, h, t, limit)
                worst = max(worst, float(np.abs(got[b, h, t] - want).max()))
    assert worst <= FP32_BOUND, f"max error {worst:.3e}"
    # The whole batch against the oracle (the reference's fp32 CPU arithmetic).
    want = O.attention_bhld(qn, kn, vn, lengths=np.array(lengths, np.int32) if lengths else None, block=block)
    assert np.abs(got - want).max() <= 1e-5
