"""GPU parity of Ops::gelu (omni_b200_gelu; semantics of src/cpu.cpp:91-96):
x = r(0.5 x (1 + erf(x * 0.70710678...))), each step an fp32 operation.

The expected values are torch's evaluation of the same fp32 steps with CUDA's
erf.  The library's bf16 path looks results up in a table that it builds from
exactly that expression (common inputs from shared memory, the rest from the
full table in global memory), and its fp32 path evaluates it directly.  So
both must agree bit for bit (any NaN for NaN).
"""

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


def _expected(z):
    return 0.5 * z * (1.0 + torch.erf(z * 0.7071067811865475244))


def _same_bits(got, want):
    nan = torch.isnan(got) & torch.isnan(want)
    return (got.view(torch.int16 if got.dtype == torch.bfloat16 else torch.int32) ==
            want.view(torch.int16 if want.dtype == torch.bfloat16 else torch.int32)) | nan


def test_gelu_bf16_every_input(ob):
    """All 65,536 bf16 bit patterns in a shuffled order (table slices and the
    global fallback mixed within warps), plus 5 more so that n is not a
    multiple of 8 (the scalar tail)."""
    g = torch.Generator().manual_seed(5)
    pats = torch.arange(65536, dtype=torch.int32)[torch.randperm(65536, generator=g)]
    pats = torch.cat([pats, torch.tensor([0x3F80, 0xBF80, 0x7F80, 0xFF80, 0x0001], dtype=torch.int32)])
    x = pats.to(torch.int16).view(torch.bfloat16).cuda()
    want = _expected(x.float()).to(torch.bfloat16)
    ob.gelu_(x)
    ob.library().sync_check()
    ok = _same_bits(x, want)
    bad = (~ok).nonzero().flatten()
    assert len(bad) == 0, f"{len(bad)} inputs differ, e.g. bits {pats[bad[:5].cpu()].tolist()}"


def test_gelu_fp32(ob):
    g = torch.Generator().manual_seed(6)
    z = torch.randn(1 << 20, generator=g) * 4
    z[:4] = torch.tensor([0.0, -0.0, float("inf"), float("-inf")])
    x = z.cuda()
    want = _expected(x.clone())
    ob.gelu_(x)
    ob.library().sync_check()
    assert bool(_same_bits(x, want).all())


def test_gelu_rejects_other_dtypes(ob):
    lib = ob.library()
    x = torch.zeros(8, dtype=torch.float16, device="cuda")
    assert lib.lib.omni_b200_gelu(x.data_ptr(), 8, 2, None) == 1
