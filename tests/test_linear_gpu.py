"""GPU parity of the bf16 linear (omni_b200_linear: the tcgen05 GEMM that the
encoder graphs use for their large linears, bias and rounding in its epilogue).

Reference: the reference's bf16-profile Ops::linear (src/cpu.cpp:47-69),
y = r(x W^T + b), computed with torch in fp32 (TF32 off) and rounded once.
The GEMM's fp32 sums run in a different order than torch's, so y may differ by
one bf16 ulp where the exact value lies near a rounding boundary, and by the
fp32 summation error where the sum cancels far below its terms: the bound is
one ulp of y plus 2^-16 of the sum of |terms|, and at least 99 % of the
outputs must match exactly.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ob():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tests.conftest import load_package

    return load_package()


def _reference(x, w, b):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        acc = x.float() @ w.float().t()
        if b is not None:
            acc = acc + b.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return acc.to(torch.bfloat16)


@pytest.mark.parametrize("rows,out_f,in_f,bias", [
    (24000, 4096, 1024, True),   # audio fc1 at 16 segments (d 1024, ffn 4096)
    (24000, 1024, 4096, True),   # audio fc2
    (23328, 3456, 1152, True),   # image QKV of 32 images (d 1152)
    (3000, 4096, 1024, True),    # two segments
    (1, 8, 8, True),             # the smallest shape
    (37, 136, 72, False),        # ragged tiles in every dimension, no bias
    (257, 512, 4096, False),     # deep K
])
def test_linear_matches_reference(ob, rows, out_f, in_f, bias):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + out_f)
    x = torch.randn(rows, in_f, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(out_f, in_f, device="cuda", generator=g) * in_f ** -0.5).to(torch.bfloat16)
    b = (torch.randn(out_f, device="cuda", generator=g) * 0.5).to(torch.bfloat16) if bias else None
    got = ob.linear(x, w, b)
    ob.library().sync_check()
    want = _reference(x, w, b).float()
    terms = x.float().abs() @ w.float().abs().t()
    if b is not None:
        terms = terms + b.float().abs()
    err = (got.float() - want).abs()
    bound = 2.0 ** -7 * want.abs() + 2.0 ** -16 * terms
    assert torch.isfinite(got.float()).all()
    assert bool((err <= bound).all()), f"max error {err.max().item():.3e}"
    assert (err == 0).float().mean().item() >= 0.99


def test_linear_rejects_bad_shapes(ob):
    lib = ob.library()
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(8, 12, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(4, 8, dtype=torch.bfloat16, device="cuda")
    st = lib.lib.omni_b200_linear(x.data_ptr(), w.data_ptr(), None, y.data_ptr(), 4, 8, 12, None, 0, None)
    assert st == 1 and b"multiples of 8" in lib.lib.omni_b200_last_error()
    st = lib.lib.omni_b200_linear(x.data_ptr(), None, None, y.data_ptr(), 4, 8, 8, None, 0, None)
    assert st == 1
